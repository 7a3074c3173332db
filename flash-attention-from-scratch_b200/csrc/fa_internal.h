#pragma once
// Host/device shared definitions of the sm_100a forward kernel (torch-free).

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

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

// The CTA-pair kernel (flash_fwd_pair_sm100.cu): d = 128, baseline / opt, no split-KV.
bool pair_kernel_supports(const FwdProblem& prob, const FwdArgs& args);
cudaError_t launch_forward_pair(const FwdProblem& prob, const FwdArgs& args, cudaStream_t stream);

// Sets a kernel's dynamic shared-memory limit once per device (the attribute persists per
// device context; setting it on every launch costs host time for nothing). Templated on the
// kernel pointer itself, so every kernel instantiation keeps its own per-device record even when
// several share one signature.
template <auto Kernel>
inline cudaError_t ensure_smem_limit(int bytes) {
    static unsigned long long done_mask = 0;  // bit d: set on device d (benign race: idempotent)
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) {
        return err;
    }
    const unsigned long long bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0ull;
    if (bit != 0 && (__atomic_load_n(&done_mask, __ATOMIC_ACQUIRE) & bit) != 0) {
        return cudaSuccess;
    }
    err = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (err == cudaSuccess && bit != 0) {
        __atomic_fetch_or(&done_mask, bit, __ATOMIC_RELEASE);
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
