/* Native C caller of libfa_b200.so through its C ABI (include/fa_b200.h) -- TEST
 * INFRASTRUCTURE: it links the double-precision oracle (oracle/attention_f64.c) as its checker.
 *
 * The counterpart of the reference's standalone driver (csrc/dev/main.cu:82-188: seeded
 * inputs, a launch checked against a double-precision CPU reference, CUDA-event timing and a
 * TFLOPS line) and of its GoogleTest API suite (tests/cpp/test_flash_fwd.cu:64-83 argument
 * validation, :115-210 shapes x variants against the CPU reference), written as a plain C
 * program: no Python, no PyTorch, no C++ -- what a cgo / JNI / N-API binding would do.
 *
 *   capi_check                         the built-in case list (exit 0 when every case passes)
 *   capi_check B H N D CAUSAL VARIANT ITERS [bf16]   one case, then ITERS timed launches
 *   capi_check --validate-only         argument validation only (needs no GPU)
 *
 * Per case: fp16 inputs from a seeded generator (xorshift64* + Box-Muller), device buffers from
 * cudaMalloc, fa_flash_fwd on a created stream, the watchdog word, the output against the
 * oracle (fp32 variants: max-abs <= max(2e-3, fp16 floor + 2.5e-4) and mean-abs <= 2e-4;
 * fp16acc: max-abs <= 1e-2), and a second launch that must reproduce the output bit for bit.
 * bf16 cases (FaFwdParams.dtype = FA_DTYPE_BFLOAT16) draw bf16 values that fp16 also holds
 * exactly (magnitudes below 2^-14 set to 0), so the same oracle checks them; their bounds are
 * the fp16 ones times 8, the ratio of the two formats' unit roundoffs.
 * fp8 cases (fa_flash_fwd_fp8) quantise each tensor to e4m3 with a power-of-two descale, so the
 * dequantized values are exact in fp16 and the oracle sees exactly what the kernel multiplies;
 * the check is the fp8 contract against exact attention: relative RMS error <= 5e-2 and
 * mean-abs <= 1e-2 (P is rounded to e4m3 for the P.V MMA).
 */
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "fa_b200.h"

int oracle_attention_f64(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t heads,
                         int64_t n, int64_t d, int causal, double scale, double* out);

#define CHECK_CUDA(call)                                                                      \
    do {                                                                                      \
        cudaError_t e_ = (call);                                                              \
        if (e_ != cudaSuccess) {                                                              \
            fprintf(stderr, "%s:%d: %s: %s\n", __FILE__, __LINE__, #call, cudaGetErrorString(e_)); \
            exit(2);                                                                          \
        }                                                                                     \
    } while (0)

static uint64_t rng_state;

static double rng_uniform(void) { /* xorshift64*, 53-bit uniform in (0, 1) */
    rng_state ^= rng_state >> 12;
    rng_state ^= rng_state << 25;
    rng_state ^= rng_state >> 27;
    const uint64_t r = rng_state * 0x2545F4914F6CDD1DULL;
    return ((double)(r >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

static double rng_normal(void) { /* Box-Muller */
    const double u = rng_uniform(), w = rng_uniform();
    return sqrt(-2.0 * log(u)) * cos(6.283185307179586 * w);
}

/* binary32 -> binary16 bits, round to nearest even (normals, subnormals, overflow to inf). */
static uint16_t float_to_half_bits(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) { /* inf / nan */
        return sign | (absx > 0x7f800000u ? 0x7e00u : 0x7c00u);
    }
    if (absx >= 0x477ff000u) { /* rounds to >= 65520: inf */
        return sign | 0x7c00u;
    }
    if (absx < 0x38800000u) { /* below the smallest normal half: subnormal or zero */
        if (absx < 0x33000000u) {
            return sign;
        }
        const uint32_t man = (absx & 0x7fffffu) | 0x800000u;
        const int shift = 126 - (int)(absx >> 23); /* 14 .. 24 */
        uint32_t h = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) {
            ++h;
        }
        return sign | (uint16_t)h;
    }
    uint32_t h = ((absx - 0x38000000u) >> 13);
    const uint32_t rem = absx & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) {
        ++h;
    }
    return sign | (uint16_t)h;
}

static double half_bits_to_double(uint16_t h) {
    const int exp = (h >> 10) & 0x1f, man = h & 0x3ff;
    double v = exp == 0 ? ldexp((double)man, -24) : ldexp((double)(man | 0x400), exp - 25);
    return (h & 0x8000u) ? -v : v;
}

static double round_to_half(double x) { return half_bits_to_double(float_to_half_bits((float)x)); }

/* binary32 -> bfloat16 bits (the high half), round to nearest even; finite inputs only. */
static uint16_t float_to_bf16_bits(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t lsb = (x >> 16) & 1u;
    return (uint16_t)((x + 0x7fffu + lsb) >> 16);
}

static double bf16_bits_to_double(uint16_t b) {
    const uint32_t x = (uint32_t)b << 16;
    float f;
    memcpy(&f, &x, 4);
    return (double)f;
}

static double round_to_bf16(double x) { return bf16_bits_to_double(float_to_bf16_bits((float)x)); }

static const char* variant_name(int v);

/* binary64 -> e4m3 (bias 7, no infinities, largest finite 448), round to nearest even,
 * saturating; the value is finite. */
static uint8_t double_to_e4m3(double x) {
    const uint8_t sign = x < 0 ? 0x80u : 0u;
    const double a = fabs(x);
    if (a < ldexp(1.0, -6)) { /* subnormal: m * 2^-9 */
        return sign | (uint8_t)nearbyint(a * 512.0); /* m = 8 encodes 2^-6, the smallest normal */
    }
    int ex = 0;
    const double fr = frexp(a, &ex); /* a = fr * 2^ex, fr in [0.5, 1) */
    int e = ex - 1;
    int q = (int)nearbyint((fr * 2.0 - 1.0) * 8.0);
    if (q == 8) {
        q = 0;
        ++e;
    }
    int code = ((e + 7) << 3) | q;
    if (code > 0x7e) {
        code = 0x7e;
    }
    return sign | (uint8_t)code;
}

static double e4m3_to_double(uint8_t c) {
    const int e = (c >> 3) & 0xf, m = c & 7;
    const double v = e == 0 ? ldexp((double)m, -9) : ldexp(1.0 + m / 8.0, e - 7);
    return (c & 0x80u) ? -v : v;
}

/* One fp8 case through fa_flash_fwd_fp8 against the double-precision oracle. */
static int run_fp8_case(int b, int h, int n, int causal, int variant, uint64_t seed) {
    const int d = 128;
    const size_t elems = (size_t)b * h * n * d;
    uint8_t* q8[3];
    uint16_t* deq[3]; /* the dequantized values as fp16 bits (exact): the oracle's inputs */
    float descale[3];
    rng_state = seed * 0x9E3779B97F4A7C15ULL + 1;
    for (int t = 0; t < 3; ++t) {
        double* x = (double*)malloc(elems * sizeof(double));
        double amax = 0.0;
        for (size_t i = 0; i < elems; ++i) {
            x[i] = rng_normal();
            amax = fabs(x[i]) > amax ? fabs(x[i]) : amax;
        }
        const double s = ldexp(1.0, (int)ceil(log2(amax / 448.0))); /* power of two */
        descale[t] = (float)s;
        q8[t] = (uint8_t*)malloc(elems);
        deq[t] = (uint16_t*)malloc(elems * 2);
        for (size_t i = 0; i < elems; ++i) {
            q8[t][i] = double_to_e4m3(x[i] / s);
            deq[t][i] = float_to_half_bits((float)(e4m3_to_double(q8[t][i]) * s));
        }
        free(x);
    }
    void *dq, *dk, *dv, *dout, *ws;
    CHECK_CUDA(cudaMalloc(&dq, elems));
    CHECK_CUDA(cudaMalloc(&dk, elems));
    CHECK_CUDA(cudaMalloc(&dv, elems));
    CHECK_CUDA(cudaMalloc(&dout, elems * 2));
    CHECK_CUDA(cudaMemcpy(dq, q8[0], elems, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(dk, q8[1], elems, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(dv, q8[2], elems, cudaMemcpyHostToDevice));
    FaFwdParams p;
    memset(&p, 0, sizeof(p));
    p.q = dq;
    p.k = dk;
    p.v = dv;
    p.o = dout;
    p.batch = b;
    p.heads = h;
    p.seqlen = n;
    p.head_dim = d;
    p.softmax_scale = (float)(1.0 / sqrt((double)d));
    p.causal = (uint8_t)causal;
    p.variant = (uint8_t)variant;
    p.dtype = FA_DTYPE_FLOAT8_E4M3;
    uint64_t ws_bytes = 0;
    if (fa_fp8_workspace_size(&p, &ws_bytes) != FA_OK) {
        fprintf(stderr, "fa_fp8_workspace_size: %s\n", fa_last_error());
        exit(1);
    }
    CHECK_CUDA(cudaMalloc(&ws, ws_bytes));
    cudaStream_t stream;
    CHECK_CUDA(cudaStreamCreate(&stream));
    uint16_t* out = (uint16_t*)malloc(elems * 2);
    uint16_t* out2 = (uint16_t*)malloc(elems * 2);
    int failed = 0;
    for (int rep = 0; rep < 2; ++rep) {
        const int rc = fa_flash_fwd_fp8(&p, descale[0], descale[1], descale[2], ws, ws_bytes, (fa_stream_t)stream);
        if (rc != FA_OK) {
            fprintf(stderr, "fa_flash_fwd_fp8 returned %d: %s\n", rc, fa_last_error());
            exit(1);
        }
        CHECK_CUDA(cudaStreamSynchronize(stream));
        CHECK_CUDA(cudaMemcpy(rep == 0 ? out : out2, dout, elems * 2, cudaMemcpyDeviceToHost));
    }
    if (memcmp(out, out2, elems * 2) != 0) {
        fprintf(stderr, "fp8 repeat launch differs\n");
        failed = 1;
    }
    double* ref = (double*)malloc(elems * sizeof(double));
    if (ref == NULL || oracle_attention_f64(deq[0], deq[1], deq[2], (int64_t)b * h, n, d, causal,
                                            (double)p.softmax_scale, ref) != 0) {
        fprintf(stderr, "oracle: out of memory\n");
        exit(2);
    }
    double se = 0.0, sr = 0.0, sum_abs = 0.0;
    for (size_t i = 0; i < elems; ++i) {
        const double e = half_bits_to_double(out[i]) - ref[i];
        se += e * e;
        sr += ref[i] * ref[i];
        sum_abs += fabs(e);
    }
    const double rel_rms = sqrt(se / (sr > 0.0 ? sr : 1.0)), mean_abs = sum_abs / (double)elems;
    if (!(rel_rms <= 5e-2) || !(mean_abs <= 1e-2)) {
        failed = 1;
    }
    printf("B%d H%d N%d D%d %s %-8s fp8  rel-rms %.3e (bound 5e-2) mean-abs %.3e (bound 1e-2) %s\n", b, h, n, d,
           causal ? "causal" : "full  ", variant_name(variant), rel_rms, mean_abs, failed ? "FAILED" : "ok");
    free(ref);
    free(out);
    free(out2);
    for (int t = 0; t < 3; ++t) {
        free(q8[t]);
        free(deq[t]);
    }
    cudaFree(dq);
    cudaFree(dk);
    cudaFree(dv);
    cudaFree(dout);
    cudaFree(ws);
    cudaStreamDestroy(stream);
    return failed;
}

static const char* variant_name(int v) {
    return v == FA_VARIANT_BASELINE ? "baseline" : v == FA_VARIANT_OPT ? "opt" : "fp16acc";
}

/* Validation through the C ABI, before any device work (reference tests/cpp/test_flash_fwd.cu:64-83). */
static int check_validation(void) {
    FaFwdParams p;
    memset(&p, 0, sizeof(p));
    p.q = p.k = p.v = (const void*)0x10000;
    p.o = (void*)0x20000;
    p.batch = 1;
    p.heads = 1;
    p.seqlen = 64;
    p.head_dim = 96;
    p.softmax_scale = 0.1f;
    p.variant = FA_VARIANT_OPT;
    int bad = 0;
    if (fa_flash_fwd(&p, NULL) != FA_ERR_INVALID_ARGUMENT || strstr(fa_last_error(), "head_dim") == NULL) {
        fprintf(stderr, "validation: head_dim 96 not rejected (%s)\n", fa_last_error());
        bad = 1;
    }
    p.head_dim = 64;
    p.seqlen = 0;
    if (fa_flash_fwd(&p, NULL) != FA_ERR_INVALID_ARGUMENT) {
        fprintf(stderr, "validation: seqlen 0 not rejected\n");
        bad = 1;
    }
    p.seqlen = 64;
    p.q = (const void*)0x10008;
    if (fa_flash_fwd(&p, NULL) != FA_ERR_INVALID_ARGUMENT || strstr(fa_last_error(), "aligned") == NULL) {
        fprintf(stderr, "validation: misaligned q not rejected (%s)\n", fa_last_error());
        bad = 1;
    }
    p.q = (const void*)0x10000;
    p.variant = 3;
    if (fa_flash_fwd(&p, NULL) != FA_ERR_INVALID_ARGUMENT || strstr(fa_last_error(), "variant") == NULL) {
        fprintf(stderr, "validation: variant 3 not rejected (%s)\n", fa_last_error());
        bad = 1;
    }
    p.variant = FA_VARIANT_OPT;
    p.dtype = 3;
    if (fa_flash_fwd(&p, NULL) != FA_ERR_INVALID_ARGUMENT || strstr(fa_last_error(), "dtype") == NULL) {
        fprintf(stderr, "validation: dtype 3 not rejected (%s)\n", fa_last_error());
        bad = 1;
    }
    p.dtype = FA_DTYPE_FLOAT8_E4M3;
    p.head_dim = 128;
    if (fa_flash_fwd(&p, NULL) != FA_ERR_INVALID_ARGUMENT || strstr(fa_last_error(), "fa_flash_fwd_fp8") == NULL) {
        fprintf(stderr, "validation: fp8 through fa_flash_fwd not rejected (%s)\n", fa_last_error());
        bad = 1;
    }
    if (fa_flash_fwd_fp8(&p, 1.0f, 1.0f, 1.0f, NULL, 0, NULL) != FA_ERR_INVALID_ARGUMENT ||
        strstr(fa_last_error(), "workspace") == NULL) {
        fprintf(stderr, "validation: fp8 without workspace not rejected (%s)\n", fa_last_error());
        bad = 1;
    }
    p.head_dim = 64;
    p.dtype = FA_DTYPE_BFLOAT16;
    p.variant = FA_VARIANT_FP16ACC;
    if (fa_flash_fwd(&p, NULL) != FA_ERR_INVALID_ARGUMENT || strstr(fa_last_error(), "fp16acc") == NULL) {
        fprintf(stderr, "validation: bf16 fp16acc not rejected (%s)\n", fa_last_error());
        bad = 1;
    }
    printf("validation: %s\n", bad ? "FAILED" : "ok");
    return bad;
}

static int run_case(int b, int h, int n, int d, int causal, int variant, int bf16, int iters, uint64_t seed) {
    const size_t elems = (size_t)b * h * n * d, bytes = elems * 2;
    uint16_t* host[3];  /* fp16 bits: the oracle's inputs */
    uint16_t* dev_in[3];  /* the kernel's inputs: host[] itself, or the same values as bf16 bits */
    rng_state = seed * 0x9E3779B97F4A7C15ULL + 1;
    for (int t = 0; t < 3; ++t) {
        host[t] = (uint16_t*)malloc(bytes);
        dev_in[t] = bf16 ? (uint16_t*)malloc(bytes) : host[t];
        for (size_t i = 0; i < elems; ++i) {
            if (bf16) {
                uint16_t bb = float_to_bf16_bits((float)rng_normal());
                if (fabs(bf16_bits_to_double(bb)) < ldexp(1.0, -14)) {
                    bb = 0;
                }
                dev_in[t][i] = bb;
                host[t][i] = float_to_half_bits((float)bf16_bits_to_double(bb));  /* exact */
            } else {
                host[t][i] = float_to_half_bits((float)rng_normal());
            }
        }
    }
    void *dq, *dk, *dv, *dout;
    CHECK_CUDA(cudaMalloc(&dq, bytes));
    CHECK_CUDA(cudaMalloc(&dk, bytes));
    CHECK_CUDA(cudaMalloc(&dv, bytes));
    CHECK_CUDA(cudaMalloc(&dout, bytes));
    CHECK_CUDA(cudaMemcpy(dq, dev_in[0], bytes, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(dk, dev_in[1], bytes, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(dv, dev_in[2], bytes, cudaMemcpyHostToDevice));
    cudaStream_t stream;
    CHECK_CUDA(cudaStreamCreate(&stream));

    FaFwdParams p;
    memset(&p, 0, sizeof(p));
    p.q = dq;
    p.k = dk;
    p.v = dv;
    p.o = dout;
    p.batch = b;
    p.heads = h;
    p.seqlen = n;
    p.head_dim = d;
    p.softmax_scale = (float)(1.0 / sqrt((double)d));
    p.causal = (uint8_t)causal;
    p.variant = (uint8_t)variant;
    p.dtype = (uint8_t)(bf16 ? FA_DTYPE_BFLOAT16 : FA_DTYPE_FLOAT16);

    int failed = 0;
    uint16_t* out = (uint16_t*)malloc(bytes);
    uint16_t* out2 = (uint16_t*)malloc(bytes);
    int rc = fa_flash_fwd(&p, (fa_stream_t)stream);
    if (rc != FA_OK) {
        fprintf(stderr, "fa_flash_fwd returned %d: %s\n", rc, fa_last_error());
        exit(1);
    }
    CHECK_CUDA(cudaStreamSynchronize(stream));
    CHECK_CUDA(cudaMemcpy(out, dout, bytes, cudaMemcpyDeviceToHost));
    rc = fa_flash_fwd(&p, (fa_stream_t)stream);
    CHECK_CUDA(cudaStreamSynchronize(stream));
    CHECK_CUDA(cudaMemcpy(out2, dout, bytes, cudaMemcpyDeviceToHost));
    if (rc != FA_OK || memcmp(out, out2, bytes) != 0) {
        fprintf(stderr, "repeat launch differs (rc %d)\n", rc);
        failed = 1;
    }
    int dev = 0;
    uint32_t status = 0;
    CHECK_CUDA(cudaGetDevice(&dev));
    if (fa_device_status(dev, 1, &status) != FA_OK || status != 0) {
        fprintf(stderr, "watchdog status %#x\n", status);
        failed = 1;
    }

    double* ref = (double*)malloc(elems * sizeof(double));
    if (ref == NULL || oracle_attention_f64(host[0], host[1], host[2], (int64_t)b * h, n, d, causal,
                                            (double)p.softmax_scale, ref) != 0) {
        fprintf(stderr, "oracle: out of memory\n");
        exit(2);
    }
    double max_abs = 0.0, sum_abs = 0.0, floor_err = 0.0;
    for (size_t i = 0; i < elems; ++i) {
        const double got = bf16 ? bf16_bits_to_double(out[i]) : half_bits_to_double(out[i]);
        const double e = fabs(got - ref[i]);
        const double f = fabs((bf16 ? round_to_bf16(ref[i]) : round_to_half(ref[i])) - ref[i]);
        max_abs = e > max_abs ? e : max_abs;
        floor_err = f > floor_err ? f : floor_err;
        sum_abs += e;
    }
    const double mean_abs = sum_abs / (double)elems;
    const int acc16 = variant == FA_VARIANT_FP16ACC;
    const double k = bf16 ? 8.0 : 1.0;  /* bf16: the fp16 bounds times 2^-8 / 2^-11 */
    const double bound = acc16 ? 1e-2 : fmax(k * 2e-3, floor_err + k * 2.5e-4);
    if (!(max_abs <= bound) || (!acc16 && !(mean_abs <= k * 2e-4))) {
        failed = 1;
    }
    printf("B%d H%d N%d D%d %s %-8s %s max-abs %.3e (bound %.3e, %s floor %.3e) mean-abs %.3e %s\n", b, h,
           n, d, causal ? "causal" : "full  ", variant_name(variant), bf16 ? "bf16" : "fp16", max_abs, bound,
           bf16 ? "bf16" : "fp16", floor_err, mean_abs, failed ? "FAILED" : "ok");

    if (iters > 0 && !failed) {
        cudaEvent_t e0, e1;
        CHECK_CUDA(cudaEventCreate(&e0));
        CHECK_CUDA(cudaEventCreate(&e1));
        for (int i = 0; i < 3; ++i) {
            fa_flash_fwd(&p, (fa_stream_t)stream);
        }
        CHECK_CUDA(cudaEventRecord(e0, stream));
        for (int i = 0; i < iters; ++i) {
            fa_flash_fwd(&p, (fa_stream_t)stream);
        }
        CHECK_CUDA(cudaEventRecord(e1, stream));
        CHECK_CUDA(cudaEventSynchronize(e1));
        float ms = 0.0f;
        CHECK_CUDA(cudaEventElapsedTime(&ms, e0, e1));
        const double flops = 4.0 * b * h * (double)n * n * d / (causal ? 2.0 : 1.0);
        printf("  %d launches: %.4f ms each, %.1f TFLOPS\n", iters, ms / iters, flops / (ms / iters * 1e-3) / 1e12);
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
    }

    free(ref);
    free(out);
    free(out2);
    for (int t = 0; t < 3; ++t) {
        if (dev_in[t] != host[t]) {
            free(dev_in[t]);
        }
        free(host[t]);
    }
    cudaFree(dq);
    cudaFree(dk);
    cudaFree(dv);
    cudaFree(dout);
    cudaStreamDestroy(stream);
    return failed;
}

int main(int argc, char** argv) {
    int failed = check_validation();
    if (argc == 2 && strcmp(argv[1], "--validate-only") == 0) {
        return failed ? 1 : 0;
    }
    if (argc == 8 || argc == 9) {
        failed |= run_case(atoi(argv[1]), atoi(argv[2]), atoi(argv[3]), atoi(argv[4]), atoi(argv[5]),
                           atoi(argv[6]), argc == 9 && strcmp(argv[8], "bf16") == 0, atoi(argv[7]), 42);
    } else if (argc == 1) {
        static const int cases[][7] = {
            /* B, H, N, D, causal, variant, bf16 */
            {1, 2, 300, 128, 1, FA_VARIANT_OPT, 0},     {2, 3, 257, 64, 0, FA_VARIANT_BASELINE, 0},
            {1, 2, 1000, 128, 1, FA_VARIANT_FP16ACC, 0}, {1, 1, 1, 64, 0, FA_VARIANT_OPT, 0},
            {2, 2, 513, 128, 0, FA_VARIANT_OPT, 0},     {1, 3, 640, 64, 1, FA_VARIANT_FP16ACC, 0},
            {1, 1, 2500, 128, 0, FA_VARIANT_BASELINE, 0}, {1, 2, 700, 128, 1, FA_VARIANT_OPT, 1},
            {2, 2, 385, 64, 0, FA_VARIANT_BASELINE, 1},
        };
        for (size_t i = 0; i < sizeof(cases) / sizeof(cases[0]); ++i) {
            const int* c = cases[i];
            failed |= run_case(c[0], c[1], c[2], c[3], c[4], c[5], c[6], 0, 1234 + i);
        }
        failed |= run_fp8_case(1, 2, 700, 1, FA_VARIANT_OPT, 77);
        failed |= run_fp8_case(2, 1, 385, 0, FA_VARIANT_BASELINE, 78);
    } else {
        fprintf(stderr, "usage: %s [B H N D CAUSAL VARIANT ITERS [bf16]]\n", argv[0]);
        return 2;
    }
    printf("capi_check: %s\n", failed ? "FAILED" : "all cases passed");
    return failed ? 1 : 0;
}
