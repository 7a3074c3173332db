/* Double-precision CPU attention -- TEST INFRASTRUCTURE ONLY (never linked into the product).
 *
 * An independent restatement of the exact attention the reference checks its kernel against
 * in C++: cpu_attention (tests/cpp/test_flash_fwd.cu:115-152) and reference_row
 * (csrc/dev/main.cu:31-63) of aligoldenhat/flash-attention-from-scratch:
 *   for every head and query row i: s_j = (q_i . k_j) * scale for j <= i (causal) or all j,
 *   p_j = exp(s_j - max_j s_j), out_i = sum_j (p_j / sum p) v_j,
 * with fp16 inputs widened exactly to double. Used for small cases as a second oracle,
 * independent of numpy's float32 arithmetic.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* IEEE-754 binary16 -> double, exact (normals, subnormals, zero, inf, nan). */
static double half_bits_to_double(uint16_t h) {
    const int sign = (h >> 15) & 1;
    const int exp = (h >> 10) & 0x1f;
    const int man = h & 0x3ff;
    double v;
    if (exp == 0) {
        v = ldexp((double)man, -24);
    } else if (exp == 31) {
        v = man ? NAN : INFINITY;
    } else {
        v = ldexp((double)(man | 0x400), exp - 25);
    }
    return sign ? -v : v;
}

/* q, k, v: [heads][n][d] binary16 bit patterns; out: [heads][n][d] double. Returns 0, or -1
 * if scratch memory could not be allocated. */
int oracle_attention_f64(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t heads,
                         int64_t n, int64_t d, int causal, double scale, double* out) {
    double* scores = (double*)malloc(sizeof(double) * (size_t)(n > 0 ? n : 1));
    double* qrow = (double*)malloc(sizeof(double) * (size_t)(d > 0 ? d : 1));
    if (scores == NULL || qrow == NULL) {
        free(scores);
        free(qrow);
        return -1;
    }
    for (int64_t h = 0; h < heads; ++h) {
        const int64_t base = h * n * d;
        for (int64_t i = 0; i < n; ++i) {
            const int64_t kv_end = causal ? i + 1 : n;
            for (int64_t c = 0; c < d; ++c) {
                qrow[c] = half_bits_to_double(q[base + i * d + c]);
            }
            double mx = -INFINITY;
            for (int64_t j = 0; j < kv_end; ++j) {
                double dot = 0.0;
                const uint16_t* kr = k + base + j * d;
                for (int64_t c = 0; c < d; ++c) {
                    dot += qrow[c] * half_bits_to_double(kr[c]);
                }
                scores[j] = dot * scale;
                if (scores[j] > mx) {
                    mx = scores[j];
                }
            }
            double sum = 0.0;
            for (int64_t j = 0; j < kv_end; ++j) {
                scores[j] = exp(scores[j] - mx);
                sum += scores[j];
            }
            double* orow = out + base + i * d;
            memset(orow, 0, sizeof(double) * (size_t)d);
            for (int64_t j = 0; j < kv_end; ++j) {
                const double p = scores[j] / sum;
                const uint16_t* vr = v + base + j * d;
                for (int64_t c = 0; c < d; ++c) {
                    orow[c] += p * half_bits_to_double(vr[c]);
                }
            }
        }
    }
    free(scores);
    free(qrow);
    return 0;
}
