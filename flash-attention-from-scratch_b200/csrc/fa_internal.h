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
};

// Variant ids as in the reference (csrc/flash_fwd.h:12-16).
enum : int { kVariantBaseline = 0, kVariantOpt = 1, kVariantFp16Acc = 2 };

// Launches the forward kernel for one (head_dim, causal, variant) on `stream`. The tensor
// maps describe q, k, v, o as [B*H][N][D] fp16 with a 64 x 128 box and 128-byte swizzle.
// Returns a cudaError_t.
cudaError_t launch_forward(int head_dim, bool causal, int variant, const CUtensorMap& tm_q,
                           const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                           const CUtensorMap& tm_o, const FwdArgs& args, cudaStream_t stream);

// Shared-memory bytes and threads per CTA of a kernel instantiation (for reports / tests).
int kernel_smem_bytes(int head_dim, bool causal, int variant);
int kernel_threads(int head_dim, bool causal, int variant);

}  // namespace fa_sm100
