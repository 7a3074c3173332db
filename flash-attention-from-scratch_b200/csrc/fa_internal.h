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

// n / d by a multiply and a shift, for 0 <= n < 2^31 and 1 <= d < 2^31 (division by an invariant
// integer, Granlund and Montgomery 1994, theorem 4.2): with l = ceil(log2 d) and
// m = ceil(2^(31+l) / d) (which fits 32 bits), floor(n / d) = floor(n m / 2^(31+l)).
// The kernel's work-item decode divides by per-launch constants on the path from one item to
// the next; this keeps each division to two dependent instructions.
struct FastDiv {
    unsigned d;
    unsigned m;
    unsigned shift;  // 31 + l

    FastDiv() : d(1), m(1u << 31), shift(31) {}
    explicit FastDiv(int divisor) {
        d = divisor > 0 ? static_cast<unsigned>(divisor) : 1u;
        unsigned l = 0;
        while ((1ull << l) < d) {
            ++l;
        }
        m = static_cast<unsigned>(((1ull << (31 + l)) + d - 1) / d);
        shift = 31 + l;
    }
    __host__ __device__ __forceinline__ int div(int n) const {
        return static_cast<int>((static_cast<unsigned long long>(static_cast<unsigned>(n)) * m) >> shift);
    }
};

struct FwdArgs {
    int seqlen;           // N (queries == keys)
    int num_bh;           // B * H
    float scale_log2;     // softmax_scale * log2(e)
    unsigned epoch;       // launch epoch, never 0
    DeviceStatus* status; // per-device watchdog record
    // Causal schedule: consecutive groups of head_group heads (the last one may be smaller);
    // each group's row blocks run longest first.
    int head_group;
    // Divisors of the work-item decode, set by the launcher: row blocks per head (nb), items per
    // key range (nb * num_bh), items per head group (nb * head_group), heads of a full group,
    // heads of the last group, key ranges of a tail block.
    FastDiv div_nb, div_per_split, div_group_items, div_group, div_last_group, div_tail;
    // Split-KV (num_splits > 1): the work item of key range z covers the z-th of num_splits
    // contiguous ranges of its row block's key tiles and writes, per row, its unnormalised fp32
    // O and (m, l) to the workspace instead of O; a combine kernel merges the ranges.
    int num_splits;       // 1 = no split
    int rows_pad;         // workspace rows per head: ceil(N / 256) * 256
    // Tail split (non-causal, num_splits == 1): items tail_from .. are the last tail_blocks row
    // blocks (in item order), each cut into tail_splits key ranges that run as separate items
    // and are merged like split-KV, so that the last partial wave of the grid takes a fraction
    // of a full item's time. tail_from == num_items: no tail split.
    int tail_from;
    int tail_blocks;
    int tail_splits;
    float* ws_o;          // split records x D fp32 (see splitkv records in the kernel)
    float* ws_ml;         // split records x 2 fp32: m (log2 units), l
    int num_items;        // work items, set by the launcher
    void* o;              // output [num_bh][seqlen][D] fp16 / bf16, set by the launcher
    float out_scale;      // fp8: O is multiplied by V's descale in the epilogue (else unused)
};

// Split-KV workspace bytes for a problem (16-byte aligned sections).
inline unsigned long long splitkv_workspace_bytes(int num_bh, int seqlen, int head_dim, int num_splits) {
    const unsigned long long rows = static_cast<unsigned long long>((seqlen + 255) / 256) * 256;
    const unsigned long long recs = rows * static_cast<unsigned long long>(num_bh) * num_splits;
    return recs * head_dim * 4ull + recs * 2ull * 4ull;
}

// The schedule of one launch, chosen at run time from (N, d, causal, variant, B * H, SMs):
// the library's counterpart of the reference's compile-time tile table
// (csrc/kernels/flash_fwd.cu:596-617), which lists runtime selection as not done
// (docs/fa3_fa4_techniques.md:29).
struct Plan {
    int rows_per_item;    // 128 x query tiles per CTA (the kernel build's NQ)
    int row_blocks;       // ceil(N / rows_per_item) * B * H
    bool persistent;      // one CTA per SM walks the items (short rows) vs one CTA per item
    int num_splits;       // key ranges of every row block (1 = none)
    int tail_blocks;      // non-causal: row blocks of the last partial wave that are cut ...
    int tail_splits;      // ... into this many key ranges (0 blocks = none)
    int head_groups;      // causal: groups of heads swept longest row block first (equal sizes
                          // ceil(B * H / head_groups), the last one possibly smaller)
    int items;            // work items
    int ctas;             // CTAs launched
    unsigned long long workspace_bytes;  // split records (0 when nothing is split)
};

// The plan for `prob` on a GPU with sm_count SMs. num_splits > 0 forces that many key ranges
// (no tail split); num_splits == 0 lets the library choose, a tail split included when
// allow_tail is set.
Plan make_plan(int num_bh, int seqlen, int head_dim, bool causal, int variant, int num_splits,
               bool allow_tail, int sm_count);

// SMs of the current device (cached per device).
int device_sm_count();

// Variant ids as in the reference (csrc/flash_fwd.h:12-16).
enum : int { kVariantBaseline = 0, kVariantOpt = 1, kVariantFp16Acc = 2 };

// One forward problem: q, k, v, o are contiguous [B*H][N][D] fp16 (bf16: bfloat16) device
// tensors.
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
    bool bf16;
    // fp8 (e4m3 q, k, v; fp16 o): vt is V transposed, [num_bh][D][vt_cols] e4m3 with keys
    // contiguous and vt_cols = seqlen rounded up to 16 (zeros beyond seqlen).
    bool fp8;
    const void* vt;
    int vt_cols;
};

// fp8: bytes of the transposed-V workspace for a problem, and the launch that fills it from V
// ([num_bh][seqlen][128] e4m3) on `stream`.
inline unsigned long long fp8_vt_bytes(int num_bh, int seqlen, int head_dim) {
    return static_cast<unsigned long long>(num_bh) * head_dim * ((seqlen + 15) / 16 * 16);
}
cudaError_t launch_fp8_transpose_v(const void* v, void* vt, int num_bh, int seqlen, cudaStream_t stream);

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

// Launches the split-KV combine over the rows of every split row block (all of them with
// num_splits > 1, the tail blocks with a tail split):
// O[bh][row] = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s, in the problem's element type.
cudaError_t launch_splitkv_combine(const FwdProblem& prob, const FwdArgs& args, const Plan& plan,
                                   cudaStream_t stream);

// Encodes the TMA tensor maps the chosen kernel needs and launches it on `stream` with the
// schedule `plan` (its split fields must match args'). Returns cudaSuccess, a CUDA launch
// error, or cudaErrorInvalidValue if a tensor map could not be encoded.
cudaError_t launch_forward(const FwdProblem& prob, const FwdArgs& args, const Plan& plan,
                           cudaStream_t stream);

// Shared-memory bytes and threads per CTA of a kernel instantiation (for reports / tests).
int kernel_smem_bytes(int head_dim, bool causal, int variant);
int kernel_threads(int head_dim, bool causal, int variant);
// Query rows per CTA (128 * query tiles per CTA).
int kernel_rows_per_cta(int head_dim, int variant);

}  // namespace fa_sm100
