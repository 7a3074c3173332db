// C entry point over the reference's own CUDA kernel (aligoldenhat/flash-attention-from-scratch,
// csrc/kernels/flash_fwd.cu, an mma.sync / ldmatrix / cp.async FlashAttention-2 kernel for
// sm_80+), compiled unmodified for sm_100a by baseline/build_ref_kernel.py. It is a context
// line for bench.py (--impl reference-kernel): the reference's GPU path on the same B200, not
// part of the product. The reference's host API is a C++ function that throws
// (csrc/flash_fwd.h:33); this shim turns that into a return code and a message.

#include <cuda_runtime.h>

#include <cstdio>
#include <exception>

#include "flash_fwd.h"

extern "C" __attribute__((visibility("default"))) int fa_ref_kernel_fwd(
    const void* q, const void* k, const void* v, void* o, int batch, int heads, int seqlen,
    int head_dim, float softmax_scale, int causal, int variant, void* stream, char* err,
    int err_len) {
    fa::FlashFwdParams p;
    p.q = q;
    p.k = k;
    p.v = v;
    p.o = o;
    p.batch = batch;
    p.heads = heads;
    p.seqlen = seqlen;
    p.head_dim = head_dim;
    p.softmax_scale = softmax_scale;
    p.causal = causal != 0;
    p.variant = static_cast<fa::Variant>(variant);
    try {
        fa::flash_fwd(p, static_cast<cudaStream_t>(stream));
    } catch (const std::exception& e) {
        if (err != nullptr && err_len > 0) {
            std::snprintf(err, static_cast<size_t>(err_len), "%s", e.what());
        }
        return 1;
    }
    return 0;
}
