#pragma once
// Softmax building blocks of the forward kernel (flash_fwd_sm100.cu).

#include <cstdint>

#include "sm100_ptx.cuh"

namespace fa_sm100 {

__device__ __forceinline__ float u2f(uint32_t x) { return __uint_as_float(x); }
__device__ __forceinline__ uint32_t f2u(float x) { return __float_as_uint(x); }

// Row max (or min, for a negative scale) of N scores (N = 64 or 128): eight independent
// three-input chains over columns 8 .. N-9, then the last eight columns.
template <bool MAX, int N>
__device__ __forceinline__ float row_extreme(const uint32_t (&sr)[N]) {
    static_assert(N % 16 == 0 && N >= 32, "row_extreme covers N = 16 k columns");
    float m[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        m[i] = u2f(sr[i]);
    }
#pragma unroll
    for (int c = 8; c + 16 <= N; c += 16) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            m[i] = MAX ? fmax3(m[i], u2f(sr[c + i]), u2f(sr[c + 8 + i]))
                       : fmin3(m[i], u2f(sr[c + i]), u2f(sr[c + 8 + i]));
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        m[i] = MAX ? fmaxf(m[i], u2f(sr[N - 8 + i])) : fminf(m[i], u2f(sr[N - 8 + i]));
    }
    return MAX ? fmax3(fmax3(m[0], m[1], m[2]), fmax3(m[3], m[4], m[5]), fmaxf(m[6], m[7]))
               : fmin3(fmin3(m[0], m[1], m[2]), fmin3(m[3], m[4], m[5]), fminf(m[6], m[7]));
}

}  // namespace fa_sm100
