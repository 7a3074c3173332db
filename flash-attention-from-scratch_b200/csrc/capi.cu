// C ABI of libfa_b200.so (declared in include/fa_b200.h): argument validation, tensor-map
// encoding, the per-device watchdog word and the head-sharding launcher.
//
// Validation mirrors the reference's fa::flash_fwd (csrc/kernels/flash_fwd.cu:625-652):
// same conditions, same messages, reported through return codes + fa_last_error() because a C
// ABI cannot throw.

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/fa_b200.h"
#include "capi_internal.h"
#include "fa_internal.h"

namespace fa_capi {

namespace {
thread_local std::string g_last_error;
}  // namespace

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

void clear_error() { g_last_error.clear(); }

const char* last_error() { return g_last_error.c_str(); }

int cuda_fail(cudaError_t err, const char* what) {
    return fail(FA_ERR_CUDA, std::string("flash_fwd: CUDA error in ") + what + ": " +
                                 cudaGetErrorString(err));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

namespace {

// One watchdog record per device, a file-scope __device__ variable; its address is looked up
// with the device current and cached for the device's current context.
__device__ fa_sm100::DeviceStatus g_device_status;

SymbolCache g_status_cache;
std::atomic<unsigned> g_epoch{0};

cudaError_t status_ptr_for(int device, fa_sm100::DeviceStatus** out) {
    void* p = nullptr;
    const cudaError_t err = g_status_cache.get(device, &p, [](void** dst) {
        return cudaGetSymbolAddress(dst, g_device_status);
    });
    *out = static_cast<fa_sm100::DeviceStatus*>(p);
    return err;
}

unsigned next_epoch() {
    unsigned e = g_epoch.fetch_add(1, std::memory_order_relaxed) + 1;
    if (e == 0) {
        e = g_epoch.fetch_add(1, std::memory_order_relaxed) + 1;
    }
    return e;
}

}  // namespace

int validate(const FaFwdParams* p) {
    if (p == nullptr) {
        return fail(FA_ERR_INVALID_ARGUMENT, "flash_fwd: params is NULL");
    }
    if (p->batch <= 0 || p->heads <= 0 || p->seqlen <= 0) {
        return fail(FA_ERR_INVALID_ARGUMENT,
                    "flash_fwd: batch, heads and seqlen must be positive");
    }
    if (static_cast<int64_t>(p->batch) * p->heads > 65535) {
        return fail(FA_ERR_INVALID_ARGUMENT,
                    "flash_fwd: batch * heads must be <= 65535 (grid.y limit)");
    }
    if (!aligned16(p->q) || !aligned16(p->k) || !aligned16(p->v) || !aligned16(p->o)) {
        return fail(FA_ERR_INVALID_ARGUMENT,
                    "flash_fwd: tensors must be 16-byte aligned (TMA)");
    }
    if (p->head_dim != 64 && p->head_dim != 128) {
        return fail(FA_ERR_INVALID_ARGUMENT, "flash_fwd: head_dim must be 64 or 128, got " +
                                                 std::to_string(p->head_dim));
    }
    if (p->variant > FA_VARIANT_FP16ACC) {
        return fail(FA_ERR_INVALID_ARGUMENT, "flash_fwd: unknown variant");
    }
    if (p->dtype > FA_DTYPE_FLOAT8_E4M3) {
        return fail(FA_ERR_INVALID_ARGUMENT,
                    "flash_fwd: dtype must be FA_DTYPE_FLOAT16, FA_DTYPE_BFLOAT16 or FA_DTYPE_FLOAT8_E4M3");
    }
    if (p->dtype == FA_DTYPE_FLOAT8_E4M3 && (p->head_dim != 128 || p->variant == FA_VARIANT_FP16ACC)) {
        return fail(FA_ERR_INVALID_ARGUMENT,
                    "flash_fwd: float8 inputs need head_dim 128 and the baseline or opt variant");
    }
    if (p->dtype == FA_DTYPE_BFLOAT16 && p->variant == FA_VARIANT_FP16ACC) {
        // kind::f16 MMAs accumulate bfloat16 products in fp32 only; the fp16 partials of
        // fp16acc need float16 operands.
        return fail(FA_ERR_INVALID_ARGUMENT, "flash_fwd: the fp16acc variant needs float16 inputs");
    }
    if (p->q == nullptr || p->k == nullptr || p->v == nullptr || p->o == nullptr) {
        return fail(FA_ERR_INVALID_ARGUMENT, "flash_fwd: null tensor pointer");
    }
    return FA_OK;
}

fa_sm100::Plan plan_for(const FaFwdParams* p, int num_splits, int sm_count) {
    if (p->dtype == FA_DTYPE_FLOAT8_E4M3) {
        num_splits = 1;  // fa_flash_fwd_fp8 never splits key ranges
    }
    return fa_sm100::make_plan(p->batch * p->heads, p->seqlen, p->head_dim, p->causal != 0, p->variant,
                               num_splits, num_splits == 0, sm_count);
}

int launch_one(const FaFwdParams* p, cudaStream_t stream, int num_splits, void* workspace,
               uint64_t workspace_bytes, const Fp8Extra* fp8) {
    const int rc = validate(p);
    if (rc != FA_OK) {
        return rc;
    }
    if ((p->dtype == FA_DTYPE_FLOAT8_E4M3) != (fp8 != nullptr) || (fp8 != nullptr && num_splits != 1)) {
        return fail(FA_ERR_INVALID_ARGUMENT, "flash_fwd: float8 inputs go through fa_flash_fwd_fp8");
    }
    if (num_splits < 0 || num_splits > kMaxSplits) {
        return fail(FA_ERR_INVALID_ARGUMENT, "flash_fwd_splitkv: num_splits must be in 1 .. 64, got " +
                                                 std::to_string(num_splits));
    }
    // The workspace is checked before any CUDA call (with explicit splits its size does not
    // depend on the device; device_sm_count falls back to 148 SMs without a device).
    const fa_sm100::Plan plan = plan_for(p, num_splits, fa_sm100::device_sm_count());
    if (plan.workspace_bytes > 0 &&
        (workspace == nullptr || workspace_bytes < plan.workspace_bytes || !aligned16(workspace))) {
        return fail(FA_ERR_INVALID_ARGUMENT,
                    std::string(num_splits == 0 ? "flash_fwd_auto" : "flash_fwd_splitkv") +
                        ": workspace must be 16-byte aligned and hold at least " +
                        std::to_string(plan.workspace_bytes) + " bytes");
    }
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) {
        return cuda_fail(err, "cudaGetDevice");
    }
    fa_sm100::DeviceStatus* status = nullptr;
    err = status_ptr_for(device, &status);
    if (err != cudaSuccess) {
        return cuda_fail(err, "cudaGetSymbolAddress");
    }
    const int bh = p->batch * p->heads;
    fa_sm100::FwdProblem prob{};
    prob.q = p->q;
    prob.k = p->k;
    prob.v = p->v;
    prob.o = p->o;
    prob.num_bh = bh;
    prob.seqlen = p->seqlen;
    prob.head_dim = p->head_dim;
    prob.causal = p->causal != 0;
    prob.variant = p->variant;
    prob.bf16 = p->dtype == FA_DTYPE_BFLOAT16;
    prob.fp8 = fp8 != nullptr;
    prob.vt = prob.fp8 ? fp8->vt : nullptr;
    prob.vt_cols = (p->seqlen + 15) / 16 * 16;
    fa_sm100::FwdArgs args{};
    args.seqlen = p->seqlen;
    args.num_bh = bh;
    // fp8: the scores of the e4m3 values carry q_descale * k_descale.
    const double qk_descale = prob.fp8 ? static_cast<double>(fp8->q_descale) * fp8->k_descale : 1.0;
    args.scale_log2 = static_cast<float>(static_cast<double>(p->softmax_scale) * qk_descale * M_LOG2E);
    args.out_scale = prob.fp8 ? fp8->v_descale : 1.0f;
    args.epoch = next_epoch();
    args.status = status;
    args.rows_pad = (p->seqlen + 255) / 256 * 256;
    if (plan.workspace_bytes > 0) {
        const uint64_t records = plan.workspace_bytes / (static_cast<uint64_t>(p->head_dim + 2) * 4u);
        args.ws_o = static_cast<float*>(workspace);
        args.ws_ml = args.ws_o + records * p->head_dim;
    }
    if (prob.fp8) {
        err = fa_sm100::launch_fp8_transpose_v(p->v, fp8->vt, bh, p->seqlen, stream);
        if (err != cudaSuccess) {
            return cuda_fail(err, "fp8 V transpose launch");
        }
    }
    err = fa_sm100::launch_forward(prob, args, plan, stream);
    if (err == cudaErrorInvalidValue) {
        return fail(FA_ERR_CUDA, "flash_fwd: cuTensorMapEncodeTiled failed");
    }
    if (err != cudaSuccess) {
        return cuda_fail(err, "kernel launch");
    }
    if (plan.workspace_bytes > 0) {
        err = fa_sm100::launch_splitkv_combine(prob, args, plan, stream);
        if (err != cudaSuccess) {
            return cuda_fail(err, "split-KV combine launch");
        }
    }
    clear_error();
    return FA_OK;
}

}  // namespace fa_capi

using fa_capi::cuda_fail;
using fa_capi::fail;
using fa_capi::launch_one;
using fa_capi::validate;

extern "C" {

int fa_flash_fwd(const FaFwdParams* params, fa_stream_t stream) {
    return launch_one(params, reinterpret_cast<cudaStream_t>(stream), 1, nullptr, 0);
}

int fa_flash_fwd_sharded(const FaFwdParams* shards, const int32_t* devices,
                         const fa_stream_t* streams, int32_t num_shards) {
    if (num_shards < 0 || (num_shards > 0 && (shards == nullptr || devices == nullptr))) {
        return fail(FA_ERR_INVALID_ARGUMENT, "flash_fwd_sharded: bad shard list");
    }
    int prev = 0;
    cudaError_t err = cudaGetDevice(&prev);
    if (err != cudaSuccess) {
        return cuda_fail(err, "cudaGetDevice");
    }
    int rc = FA_OK;
    for (int i = 0; i < num_shards && rc == FA_OK; ++i) {
        err = cudaSetDevice(devices[i]);
        if (err != cudaSuccess) {
            rc = cuda_fail(err, "cudaSetDevice");
            break;
        }
        rc = launch_one(&shards[i],
                        streams != nullptr ? reinterpret_cast<cudaStream_t>(streams[i]) : nullptr, 1,
                        nullptr, 0);
    }
    cudaSetDevice(prev);
    return rc;
}

const char* fa_last_error(void) { return fa_capi::last_error(); }

int fa_device_status(int32_t device, int32_t clear, uint32_t* status_out) {
    int prev = 0;
    cudaError_t err = cudaGetDevice(&prev);
    if (err != cudaSuccess) {
        return cuda_fail(err, "cudaGetDevice");
    }
    err = cudaSetDevice(device);
    if (err != cudaSuccess) {
        return cuda_fail(err, "cudaSetDevice");
    }
    fa_sm100::DeviceStatus* ptr = nullptr;
    fa_sm100::DeviceStatus host{};
    err = fa_capi::status_ptr_for(device, &ptr);
    if (err == cudaSuccess) {
        err = cudaDeviceSynchronize();
    }
    if (err == cudaSuccess) {
        err = cudaMemcpy(&host, ptr, sizeof(host), cudaMemcpyDeviceToHost);
    }
    if (err == cudaSuccess && clear != 0) {
        const fa_sm100::DeviceStatus zero{};
        err = cudaMemcpy(ptr, &zero, sizeof(zero), cudaMemcpyHostToDevice);
    }
    cudaSetDevice(prev);
    if (err != cudaSuccess) {
        return cuda_fail(err, "fa_device_status");
    }
    if (status_out != nullptr) {
        *status_out = host.code;
    }
    return FA_OK;
}

int fa_splitkv_workspace_size(const FaFwdParams* params, int32_t num_splits, uint64_t* bytes_out) {
    const int rc = validate(params);
    if (rc != FA_OK) {
        return rc;
    }
    if (num_splits < 1 || num_splits > fa_capi::kMaxSplits) {
        return fail(FA_ERR_INVALID_ARGUMENT, "flash_fwd_splitkv: num_splits must be in 1 .. 64, got " +
                                                 std::to_string(num_splits));
    }
    if (bytes_out != nullptr) {
        *bytes_out = num_splits == 1 ? 0
                                     : fa_sm100::splitkv_workspace_bytes(params->batch * params->heads,
                                                                         params->seqlen, params->head_dim,
                                                                         num_splits);
    }
    fa_capi::clear_error();
    return FA_OK;
}

int fa_splitkv_choose(const FaFwdParams* params, int32_t num_sms, int32_t* num_splits_out) {
    const int rc = validate(params);
    if (rc != FA_OK) {
        return rc;
    }
    if (num_sms <= 0) {
        return fail(FA_ERR_INVALID_ARGUMENT, "flash_fwd_splitkv: num_sms must be positive");
    }
    if (num_splits_out != nullptr) {
        *num_splits_out = fa_capi::plan_for(params, 0, num_sms).num_splits;
    }
    fa_capi::clear_error();
    return FA_OK;
}

int fa_plan(const FaFwdParams* params, int32_t num_sms, FaPlan* plan_out) {
    const int rc = validate(params);
    if (rc != FA_OK) {
        return rc;
    }
    const fa_sm100::Plan p = fa_capi::plan_for(params, 0, num_sms > 0 ? num_sms : fa_sm100::device_sm_count());
    if (plan_out != nullptr) {
        plan_out->rows_per_item = p.rows_per_item;
        plan_out->persistent = p.persistent ? 1 : 0;
        plan_out->num_splits = p.num_splits;
        plan_out->tail_blocks = p.tail_blocks;
        plan_out->tail_splits = p.tail_splits;
        plan_out->head_groups = p.head_groups;
        plan_out->items = p.items;
        plan_out->ctas = p.ctas;
        plan_out->workspace_bytes = p.workspace_bytes;
    }
    fa_capi::clear_error();
    return FA_OK;
}

int fa_flash_fwd_auto(const FaFwdParams* params, void* workspace, uint64_t workspace_bytes,
                      fa_stream_t stream) {
    return launch_one(params, reinterpret_cast<cudaStream_t>(stream), 0, workspace, workspace_bytes);
}

int fa_flash_fwd_splitkv(const FaFwdParams* params, int32_t num_splits, void* workspace,
                         uint64_t workspace_bytes, fa_stream_t stream) {
    if (params != nullptr && validate(params) == FA_OK && (num_splits < 1 || num_splits > fa_capi::kMaxSplits)) {
        return fail(FA_ERR_INVALID_ARGUMENT, "flash_fwd_splitkv: num_splits must be in 1 .. 64, got " +
                                                 std::to_string(num_splits));
    }
    return launch_one(params, reinterpret_cast<cudaStream_t>(stream), num_splits, workspace,
                      workspace_bytes);
}

int fa_fp8_workspace_size(const FaFwdParams* params, uint64_t* bytes_out) {
    const int rc = validate(params);
    if (rc != FA_OK) {
        return rc;
    }
    if (params->dtype != FA_DTYPE_FLOAT8_E4M3) {
        return fail(FA_ERR_INVALID_ARGUMENT, "flash_fwd_fp8: params->dtype must be FA_DTYPE_FLOAT8_E4M3");
    }
    if (bytes_out != nullptr) {
        *bytes_out = fa_sm100::fp8_vt_bytes(params->batch * params->heads, params->seqlen, params->head_dim);
    }
    fa_capi::clear_error();
    return FA_OK;
}

int fa_flash_fwd_fp8(const FaFwdParams* params, float q_descale, float k_descale, float v_descale,
                     void* workspace, uint64_t workspace_bytes, fa_stream_t stream) {
    uint64_t need = 0;
    const int rc = fa_fp8_workspace_size(params, &need);
    if (rc != FA_OK) {
        return rc;
    }
    if (!(q_descale > 0.0f) || !(k_descale > 0.0f) || !(v_descale > 0.0f) || !std::isfinite(q_descale) ||
        !std::isfinite(k_descale) || !std::isfinite(v_descale)) {
        return fail(FA_ERR_INVALID_ARGUMENT, "flash_fwd_fp8: descales must be positive and finite");
    }
    if (workspace == nullptr || workspace_bytes < need || !fa_capi::aligned16(workspace)) {
        return fail(FA_ERR_INVALID_ARGUMENT, "flash_fwd_fp8: workspace must be 16-byte aligned and hold at least " +
                                                 std::to_string(need) + " bytes");
    }
    const fa_capi::Fp8Extra extra{q_descale, k_descale, v_descale, workspace};
    return launch_one(params, reinterpret_cast<cudaStream_t>(stream), 1, nullptr, 0, &extra);
}

int fa_kernel_info(int32_t head_dim, int32_t variant, int32_t* smem_bytes, int32_t* threads) {
    if ((head_dim != 64 && head_dim != 128) || variant < 0 || variant > FA_VARIANT_FP16ACC) {
        return fail(FA_ERR_INVALID_ARGUMENT, "fa_kernel_info: bad head_dim or variant");
    }
    if (smem_bytes != nullptr) {
        *smem_bytes = fa_sm100::kernel_smem_bytes(head_dim, false, variant);
    }
    if (threads != nullptr) {
        *threads = fa_sm100::kernel_threads(head_dim, false, variant);
    }
    return FA_OK;
}

}  // extern "C"
