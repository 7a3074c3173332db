#pragma once
// Host/device shared definitions of the sm_100a forward kernel (torch-free).

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

namespace fa_sm100 {

// Device-side watchdog record. `code` accumulates kStatus* bits of every launch that gave up
// a wait (sticky until the host clears it); `epoch_aborted` holds the launch epoch of the most
// recent launch that gave up, so that the remaining CTAs of that launch stop quickly while
// later launches are unaffected.
struct DeviceStatus {
    unsigned code;
    unsigned epoch_aborted;
};

struct FwdArgs {
    int seqlen;           // N (queries == keys)
    int num_bh;           // B * H
    float scale_log2;     // softmax_scale * log2(e)
    unsigned epoch;       // launch epoch, never 0
    DeviceStatus* status; // per-device watchdog record
    int head_group;       // causal schedule: heads interleaved in one heavy-first sweep (>= 1)
    // Split-KV (num_splits > 1): the work item of key range z covers the z-th of num_splits
    // contiguous ranges of its row block's key tiles and writes, per row, its unnormalised fp32
    // O and (m, l) to the workspace instead of O; a combine kernel merges the ranges.
    int num_splits;       // 1 = no split
    int rows_pad;         // workspace rows per head: ceil(N / 256) * 256
    float* ws_o;          // [num_splits][num_bh][rows_pad][D] fp32
    float* ws_ml;         // [num_splits][num_bh][rows_pad][2] fp32: m (log2 units), l
    int num_items;        // work items (row blocks x heads x key ranges), set by the launcher
    void* o;              // output [num_bh][seqlen][D] fp16, set by the launcher
};

// Split-KV workspace bytes for a problem (16-byte aligned sections).
inline unsigned long long splitkv_workspace_bytes(int num_bh, int seqlen, int head_dim, int num_splits) {
    const unsigned long long rows = static_cast<unsigned long long>((seqlen + 255) / 256) * 256;
    const unsigned long long recs = rows * static_cast<unsigned long long>(num_bh) * num_splits;
    return recs * head_dim * 4ull + recs * 2ull * 4ull;
}

// Variant ids as in the reference (csrc/flash_fwd.h:12-16).
enum : int { kVariantBaseline = 0, kVariantOpt = 1, kVariantFp16Acc = 2 };

// One forward problem: q, k, v, o are contiguous [B*H][N][D] fp16 device tensors.
struct FwdProblem {
    const void* q;
    const void* k;
    const void* v;
    void* o;
    int num_bh;
    int seqlen;
    int head_dim;
    bool causal;
    int variant;
};

// Unique id (cuCtxGetId, plus one) of the calling thread's current CUDA context, or 0 when
// no context is current or the driver lacks the call. Values the library caches per device
// (device addresses of module variables, kernel attributes that were set) belong to one
// context: a device reset destroys the primary context and a new one replaces it, so every
// such cache keys its entries on this id and refills them when it changes.
inline unsigned long long current_context_id() {
    static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
    static PFN_cuCtxGetId_v12000 get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 4000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
        }
        p = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
        }
    });
    CUcontext ctx = nullptr;
    if (get_current == nullptr || get_id == nullptr || get_current(&ctx) != CUDA_SUCCESS ||
        ctx == nullptr) {
        return 0;
    }
    unsigned long long id = 0;
    return get_id(ctx, &id) == CUDA_SUCCESS ? id + 1 : 0;
}

// Sets a kernel's dynamic shared-memory limit once per device context (the attribute persists
// in the context; setting it on every launch costs host time for nothing). Templated on the
// kernel pointer itself, so every kernel instantiation keeps its own per-device record even when
// several share one signature.
template <auto Kernel>
inline cudaError_t ensure_smem_limit(int bytes) {
    static unsigned long long done_ctx[64] = {};  // context id per device where it is set
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) {
        return err;
    }
    const bool tracked = dev >= 0 && dev < 64;
    const unsigned long long ctx = current_context_id();
    if (tracked && ctx != 0 && __atomic_load_n(&done_ctx[dev], __ATOMIC_ACQUIRE) == ctx) {
        return cudaSuccess;
    }
    err = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (err == cudaSuccess && tracked) {
        // The call above made the device's context current if none was.
        __atomic_store_n(&done_ctx[dev], current_context_id(), __ATOMIC_RELEASE);
    }
    return err;
}

// Launches the split-KV combine: O[bh][row] = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s, fp16.
cudaError_t launch_splitkv_combine(const FwdProblem& prob, const FwdArgs& args, cudaStream_t stream);

// Encodes the TMA tensor maps the chosen kernel needs and launches it on `stream`.
// Returns cudaSuccess, a CUDA launch error, or cudaErrorInvalidValue if a tensor map could not
// be encoded.
cudaError_t launch_forward(const FwdProblem& prob, const FwdArgs& args, cudaStream_t stream);

// Shared-memory bytes and threads per CTA of a kernel instantiation (for reports / tests).
int kernel_smem_bytes(int head_dim, bool causal, int variant);
int kernel_threads(int head_dim, bool causal, int variant);
// Query rows per CTA (128 * query tiles per CTA).
int kernel_rows_per_cta(int head_dim, int variant);

}  // namespace fa_sm100
