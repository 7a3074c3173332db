#pragma once
// Pieces of the C ABI (include/fa_b200.h) shared by its translation units: error reporting,
// argument validation, the per-context symbol-address cache and the launch path.

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "../../include/fa_b200.h"
#include "fa_internal.h"

namespace fa_capi {

constexpr int kMaxDevices = 64;
constexpr int kMaxSplits = 64;

// Sets the calling thread's fa_last_error() message and returns `code`.
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t err, const char* what);
void clear_error();
const char* last_error();

bool aligned16(const void* p);

// The reference's fa::flash_fwd checks (csrc/kernels/flash_fwd.cu:625-652), same messages.
int validate(const FaFwdParams* p);

// The schedule for `p` on a GPU with sm_count SMs: num_splits key ranges per row block, or,
// with num_splits == 0, the library's choice (split-KV for few row blocks, a tail split of the
// last partial wave). e4m3 problems always get one key range.
fa_sm100::Plan plan_for(const FaFwdParams* p, int num_splits, int sm_count);

// fp8 launch extras: per-tensor descales and the transposed-V workspace.
struct Fp8Extra {
    float q_descale;
    float k_descale;
    float v_descale;
    void* vt;
};

// Validates, plans (num_splits as in plan_for), encodes the tensor maps and enqueues the forward
// plus, when the plan splits key ranges, the combine, with `workspace` holding the partials.
// e4m3 inputs (p->dtype == FA_DTYPE_FLOAT8_E4M3) need `fp8` (and num_splits == 1); the
// transpose of V into fp8->vt is enqueued first.
int launch_one(const FaFwdParams* p, cudaStream_t stream, int num_splits, void* workspace,
               uint64_t workspace_bytes, const Fp8Extra* fp8 = nullptr);

// Device address of a module variable, looked up per device with that device current and
// cached for the device's current context (a device reset replaces the context, which voids
// the address; the next lookup then refills the entry).
class SymbolCache {
public:
    // `lookup` is called with the device current and must store the address in *out.
    template <class Lookup>
    cudaError_t get(int device, void** out, Lookup lookup) {
        if (device < 0 || device >= kMaxDevices) {
            return cudaErrorInvalidDevice;
        }
        std::lock_guard<std::mutex> lock(mutex_);
        const unsigned long long ctx = fa_sm100::current_context_id();
        if (ptr_[device] == nullptr || ctx == 0 || ctx != ctx_[device]) {
            void* p = nullptr;
            const cudaError_t err = lookup(&p);
            if (err != cudaSuccess) {
                return err;
            }
            ptr_[device] = p;
            ctx_[device] = fa_sm100::current_context_id();  // the lookup made a context current
        }
        *out = ptr_[device];
        return cudaSuccess;
    }

private:
    std::mutex mutex_;
    void* ptr_[kMaxDevices] = {};
    unsigned long long ctx_[kMaxDevices] = {};
};

}  // namespace fa_capi
