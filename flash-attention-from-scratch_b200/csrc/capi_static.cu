// fa_flash_fwd_splitkv_static (include/fa_b200.h): split-KV whose partials go to a fixed
// scratch array of this library instead of a caller workspace, so the call allocates nothing.
// No counterpart in the reference.
//
// The array lives in this translation unit, i.e. in a module of its own: with CUDA's lazy
// module loading (the default since CUDA 12.2) a device reserves its 32 MiB only once this
// entry point has been called there; with CUDA_MODULE_LOADING=EAGER every device the process
// uses for the library reserves it at context creation. Either way it stays reserved until
// the process exits.

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "../../include/fa_b200.h"
#include "capi_internal.h"
#include "fa_internal.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t{32} << 20;
static __device__ __align__(256) unsigned char g_splitkv_scratch[kStaticScratchBytes];

// In host code `g_splitkv_scratch` names a host-side stand-in, not device memory: the device
// address comes from cudaGetSymbolAddress with the device current, cached for the device's
// current context.
fa_capi::SymbolCache g_scratch_cache;

cudaError_t scratch_ptr_for(int device, void** out) {
    return g_scratch_cache.get(device, out, [](void** dst) {
        return cudaGetSymbolAddress(dst, g_splitkv_scratch);
    });
}

}  // namespace

extern "C" {

int fa_flash_fwd_splitkv_static(const FaFwdParams* params, int32_t num_splits, fa_stream_t stream) {
    using fa_capi::fail;
    const int rc = fa_capi::validate(params);
    if (rc != FA_OK) {
        return rc;
    }
    if (num_splits < 1 || num_splits > fa_capi::kMaxSplits) {
        return fail(FA_ERR_INVALID_ARGUMENT,
                    "flash_fwd_splitkv_static: num_splits must be in 1 .. 64, got " +
                        std::to_string(num_splits));
    }
    const uint64_t need =
        num_splits == 1 ? 0
                        : fa_sm100::splitkv_workspace_bytes(params->batch * params->heads,
                                                            params->seqlen, params->head_dim, num_splits);
    if (need > kStaticScratchBytes) {
        return fail(FA_ERR_INVALID_ARGUMENT,
                    "flash_fwd_splitkv_static: the problem needs " + std::to_string(need) +
                        " bytes of scratch; the static scratch holds " +
                        std::to_string(kStaticScratchBytes) +
                        " (use fa_flash_fwd_splitkv with a caller workspace)");
    }
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) {
        return fa_capi::cuda_fail(err, "cudaGetDevice");
    }
    void* scratch = nullptr;
    err = scratch_ptr_for(device, &scratch);
    if (err != cudaSuccess) {
        return fa_capi::cuda_fail(err, "cudaGetSymbolAddress");
    }
    return fa_capi::launch_one(params, reinterpret_cast<cudaStream_t>(stream), num_splits, scratch,
                               kStaticScratchBytes);
}

}  // extern "C"
