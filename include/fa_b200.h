/* C ABI of the B200 (sm_100a) FlashAttention-2 forward library, libfa_b200.so.
 *
 * Plain C: raw device pointers, sizes and a CUDA stream handle, no PyTorch or C++ types, so a
 * ctypes / cgo / JNI / N-API binding can call it directly. The library allocates no device
 * memory. Every entry point is re-entrant and thread-safe and keeps no per-call state, with one
 * exception: fa_flash_fwd_splitkv_static shares one fixed scratch per device between its calls
 * (see its declaration). Device addresses and kernel attributes the library caches are keyed
 * on the device's current CUDA context, so they are looked up again after a device reset.
 *
 * Reference interfaces each entry point replaces (aligoldenhat/flash-attention-from-scratch):
 *   FaFwdParams          <- fa::FlashFwdParams          csrc/flash_fwd.h:18-30
 *   FA_VARIANT_*         <- fa::Variant                 csrc/flash_fwd.h:12-16
 *   fa_flash_fwd()       <- fa::flash_fwd()             csrc/flash_fwd.h:32-33,
 *                                                       csrc/kernels/flash_fwd.cu:625-652
 *   fa_last_error()      <- the what() string of the std::invalid_argument / runtime_error
 *                           that fa::flash_fwd throws (csrc/kernels/flash_fwd.cu:626-651,
 *                           csrc/common.cuh:15-26); a C ABI cannot throw.
 */
#ifndef FA_B200_H_
#define FA_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define FA_API __attribute__((visibility("default")))
#else
#define FA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same layout as cudaStream_t / CUstream; NULL is the legacy default stream. */
struct CUstream_st;
typedef struct CUstream_st* fa_stream_t;

/* Return codes. */
#define FA_OK 0
#define FA_ERR_INVALID_ARGUMENT 1 /* reference: std::invalid_argument (Python ValueError) */
#define FA_ERR_CUDA 2             /* reference: std::runtime_error from CUDA_CHECK        */
#define FA_ERR_DEVICE_TIMEOUT 3   /* a kernel gave up a bounded wait (see fa_device_status) */

/* Kernel builds (reference csrc/flash_fwd.h:12-16). */
#define FA_VARIANT_BASELINE 0 /* exact running max, fp32 accumulation                      */
#define FA_VARIANT_OPT 1      /* lazy rescale (threshold 2^8), fp32 accumulation (default)  */
#define FA_VARIANT_FP16ACC 2  /* P.V accumulated in fp16 per key tile, folded into fp32     */

/* Element type of q, k, v and o (FaFwdParams.dtype). The reference takes float16 only
 * (csrc/bindings.cpp:34); bfloat16 is an extension (its docs/fa3_fa4_techniques.md:22,90 list
 * bf16 inputs as not done) that runs the baseline and opt variants, with P rounded to bfloat16
 * for the P.V MMA and fp32 accumulation; FA_VARIANT_FP16ACC needs float16. */
#define FA_DTYPE_FLOAT16 0
#define FA_DTYPE_BFLOAT16 1
#define FA_DTYPE_FLOAT8_E4M3 2 /* q, k, v e4m3 and o float16: fa_flash_fwd_fp8 only */

/* Forward parameters (reference fa::FlashFwdParams, csrc/flash_fwd.h:18-30).
 * q, k, v, o: [batch, heads, seqlen, head_dim] of `dtype` (float16 unless set; all four the
 * same type), contiguous, 16-byte aligned, on the current CUDA device. o is written; the
 * caller owns every buffer. */
typedef struct FaFwdParams {
    const void* q;
    const void* k;
    const void* v;
    void* o;
    int32_t batch;
    int32_t heads;
    int32_t seqlen;   /* N, queries == keys */
    int32_t head_dim; /* 64 or 128 */
    float softmax_scale;
    uint8_t causal;
    uint8_t variant; /* FA_VARIANT_* */
    uint8_t dtype;   /* FA_DTYPE_* (0, float16, in a zero-initialised struct) */
    uint8_t reserved;
} FaFwdParams;

/* Enqueues O = softmax(Q K^T * scale) V on `stream` (current device), one range of keys per
 * row block (fa_flash_fwd_auto may split key ranges). Asynchronous: no host synchronisation.
 * Validates like the reference (batch, heads, seqlen > 0; head_dim 64/128; batch*heads <=
 * 65535; 16-byte aligned pointers; known variant), plus a known dtype (float16 for
 * FA_VARIANT_FP16ACC), and returns FA_ERR_INVALID_ARGUMENT with a message in fa_last_error()
 * on failure.
 * Reference: fa::flash_fwd, csrc/kernels/flash_fwd.cu:625-652. */
FA_API int fa_flash_fwd(const FaFwdParams* params, fa_stream_t stream);

/* Host-side head-sharding launcher: shard i is enqueued on device devices[i] and stream
 * streams[i] (each shard a complete [b, h, N, d] problem already resident on that device).
 * No collective: heads are independent. Returns the first error; later shards are not
 * launched after an error. Replaces the single-GPU launch loop of bench/benchmark.py:108-120
 * for multi-GPU runs (the reference has no multi-GPU code). */
FA_API int fa_flash_fwd_sharded(const FaFwdParams* shards, const int32_t* devices,
                         const fa_stream_t* streams, int32_t num_shards);

/* Message of the last error on the calling thread ("" if none). */
FA_API const char* fa_last_error(void);

/* Reads (and if clear != 0, clears) the sticky device watchdog bits of `device`: nonzero
 * means a kernel gave up a bounded wait instead of hanging, and its output is not valid.
 * Synchronises the device. Returns FA_OK and writes the bits to *status_out. */
FA_API int fa_device_status(int32_t device, int32_t clear, uint32_t* status_out);

/* Shared memory bytes and threads per CTA of the kernel used for (head_dim, variant). */
FA_API int fa_kernel_info(int32_t head_dim, int32_t variant, int32_t* smem_bytes, int32_t* threads);

/* ---- Split-KV (no counterpart in the reference, which lists it as not done:
 *      docs/optimizations.md:372-373). For few heads x long N, where ceil(N / 256) * B * H
 *      CTAs leave SMs idle, each row block's key tiles are cut into num_splits contiguous
 *      ranges; every range writes its rows' unnormalised O and (max, sum) to a caller-owned
 *      workspace and a second kernel merges the ranges in index order (deterministic). */

/* Bytes of workspace fa_flash_fwd_splitkv needs for `params` and num_splits (1 .. 64):
 * num_splits * batch * heads * ceil(seqlen / 256) * 256 * (head_dim + 2) * 4. */
FA_API int fa_splitkv_workspace_size(const FaFwdParams* params, int32_t num_splits,
                                     uint64_t* bytes_out);

/* A split count for `params` on a GPU with num_sms SMs: 1 when the row blocks already fill
 * the GPU, else about num_sms / row blocks, keeping at least two key tiles per range, at most 16. */
FA_API int fa_splitkv_choose(const FaFwdParams* params, int32_t num_sms, int32_t* num_splits_out);

/* fa_flash_fwd with the key range split num_splits ways (1 = fa_flash_fwd). `workspace`:
 * device memory of at least fa_splitkv_workspace_size bytes, 16-byte aligned; it needs no
 * initialisation and may be reused once the call's work on `stream` has completed. Same
 * validation and codes as fa_flash_fwd, plus FA_ERR_INVALID_ARGUMENT for num_splits outside
 * 1 .. 64 or a missing / small / misaligned workspace. */
FA_API int fa_flash_fwd_splitkv(const FaFwdParams* params, int32_t num_splits, void* workspace,
                                uint64_t workspace_bytes, fa_stream_t stream);

/* ---- Runtime schedule selection (no counterpart in the reference, whose schedule is a
 *      compile-time tile table per (d, causal), csrc/kernels/flash_fwd.cu:596-617, and which
 *      lists runtime selection by sequence length as not done, docs/fa3_fa4_techniques.md:29). */

/* The schedule fa_flash_fwd_auto runs for a problem. */
typedef struct FaPlan {
    int32_t rows_per_item;  /* query rows per work item: 128 x query tiles per CTA (256, or 128
                               for fp16acc at head_dim 128) */
    int32_t persistent;     /* 1: a grid of one CTA per SM walks the items (rows up to 2048,
                               non-causal rows up to 8192); 0: one CTA per item */
    int32_t num_splits;     /* key ranges of every row block (split-KV); 1 = none */
    int32_t tail_blocks;    /* non-causal: row blocks of the grid's last partial wave, each cut
                               into tail_splits key ranges; 0 = none */
    int32_t tail_splits;
    int32_t head_groups;    /* causal: groups of ceil(B*H / head_groups) heads (the last one may
                               be smaller) whose row blocks run
                               longest first, each group's K and V sized to stay in L2 */
    int32_t items;          /* work items */
    int32_t ctas;           /* CTAs launched */
    uint64_t workspace_bytes; /* device workspace for the split partials (0: none needed) */
} FaPlan;

/* The schedule for `params` on a GPU with num_sms SMs (num_sms <= 0: the current device's).
 * Validates like fa_flash_fwd; makes no device allocation and launches nothing. */
FA_API int fa_plan(const FaFwdParams* params, int32_t num_sms, FaPlan* plan_out);

/* fa_flash_fwd with the library's schedule (fa_plan on the current device): split-KV when the
 * row blocks leave SMs idle, a tail split of the last partial wave for non-causal problems with
 * few waves. `workspace`: device memory of at least the plan's workspace_bytes, 16-byte aligned
 * (may be NULL when that is 0); it needs no initialisation and may be reused once the call's
 * work on `stream` has completed. Results are deterministic for a given device type. */
FA_API int fa_flash_fwd_auto(const FaFwdParams* params, void* workspace, uint64_t workspace_bytes,
                             fa_stream_t stream);

/* ---- fp8 (e4m3) inputs (no counterpart in the reference, which lists fp8 attention as not
 *      done: docs/fa3_fa4_techniques.md:22,132-138). q, k, v hold e4m3 values with one descale
 *      per tensor (the real value is the e4m3 value times its descale), o is float16; head_dim
 *      128, the baseline or opt variant (opt's lazy threshold is 2^4 here). Scores and
 *      accumulators are fp32; P is rounded to e4m3 as p * 2^(8 - threshold) (within e4m3's
 *      range) for the P.V MMA and the row sums add the rounded values. Key ranges are never
 *      split. params->dtype must be FA_DTYPE_FLOAT8_E4M3 (the other entry points reject it). */

/* Bytes of device workspace fa_flash_fwd_fp8 needs: V transposed, batch * heads * head_dim *
 * (seqlen rounded up to 16). */
FA_API int fa_fp8_workspace_size(const FaFwdParams* params, uint64_t* bytes_out);

/* O = softmax(q_descale * k_descale * softmax_scale * Q K^T) (v_descale * V), Q, K, V e4m3, O
 * float16, enqueued on `stream`: first a transpose of V into `workspace` (at least
 * fa_fp8_workspace_size bytes, 16-byte aligned, overlapping none of q, k, v and o, reusable
 * once the call's work has completed), then the forward kernel. Descales must be positive and
 * finite. */
FA_API int fa_flash_fwd_fp8(const FaFwdParams* params, float q_descale, float k_descale,
                            float v_descale, void* workspace, uint64_t workspace_bytes,
                            fa_stream_t stream);

/* fa_flash_fwd_splitkv without a caller workspace, allocating nothing (no counterpart in the
 * reference), for callers that cannot allocate device memory or hand it over (a runtime whose
 * allocator is not exposed to the binding, or a host language without CUDA bindings). The
 * split partials go to a fixed scratch of 32 MiB (33554432 bytes) per device, a static
 * __device__ array of the library; a problem whose split-KV workspace
 * (fa_splitkv_workspace_size) exceeds it is rejected with FA_ERR_INVALID_ARGUMENT and a
 * message. Nothing in the scratch needs to start at zero: every record a call reads was
 * written by the same call. The array is in a module of its own: under CUDA's lazy module
 * loading (the default) a device holds its 32 MiB from the first call of this entry point
 * there until the process exits; under CUDA_MODULE_LOADING=EAGER every device the library
 * runs on holds it, whichever entry points are called. The first call on each device (and
 * the first after a device reset) looks the scratch address up (cudaGetSymbolAddress) and
 * caches it; make that first call outside any stream capture. There is one scratch per
 * device: calls whose work can overlap on the GPU (different streams without ordering between
 * them) race on it and give wrong results; calls on one stream are ordered by the stream. */
FA_API int fa_flash_fwd_splitkv_static(const FaFwdParams* params, int32_t num_splits,
                                       fa_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FA_B200_H_ */
