/*
 * Exhaustive check of the division the LayerNorm kernels use for the Welford mean update
 * (TEST INFRASTRUCTURE ONLY).  The reference computes delta / (float)count with IEEE
 * round-to-nearest division (kernel/csrc/turing/segmented_rms_adaln.cu:262-265).  For
 * the small integer counts of the per-thread pass, the B200 kernel instead forms
 *
 *     y  = RN(1 / count)                  (a compile-time constant per unrolled step)
 *     q0 = RN(delta * y)
 *     r  = RN(delta - q0 * count)         (one fma; exact)
 *     q  = RN(q0 + r * y)                 (one fma)
 *
 * the correction step of Markstein's division (P. Markstein, "Computation of elementary
 * functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990), and
 * falls back to the IEEE division when delta is zero, not finite or below 2^-96 in
 * magnitude.  The Welford combine steps divide by larger counts (up to the row width)
 * with the same step and a reciprocal rounded at run time.  The quotient of a normal
 * delta scales exactly with delta's exponent, so one binade of delta covers every
 * exponent in the fast range; this program checks every `stride`-th significand of the
 * binades [1, 2) and [2^-96, 2^-95), both signs, for every count in first..last, against
 * C's IEEE division, and prints the number of checks and of mismatches.
 *
 *   division_check LAST [STRIDE [FIRST]]
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static float from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

int main(int argc, char **argv) {
    const int max_count = argc > 1 ? atoi(argv[1]) : 128;
    const uint32_t stride = argc > 2 ? (uint32_t)atoi(argv[2]) : 1u;  /* 1 = every significand */
    const int first = argc > 3 ? atoi(argv[3]) : 1;
    long long checked = 0, mismatches = 0;
#pragma omp parallel for reduction(+ : checked, mismatches) schedule(dynamic)
    for (int count = first; count <= max_count; ++count) {
        const float c = (float)count;
        const float y = 1.0f / c;
        const uint32_t exps[2] = {127u, 127u - 96u};
        for (int e = 0; e < 2; ++e) {
            for (uint32_t m = 0; m < (1u << 23); m += stride) {
                for (uint32_t sign = 0; sign < 2; ++sign) {
                    const float delta = from_bits((sign << 31) | (exps[e] << 23) | m);
                    const float want = delta / c;
                    const float q0 = delta * y;
                    const float r = fmaf(-q0, c, delta);
                    const float q = fmaf(r, y, q0);
                    ++checked;
                    if (to_bits(q) != to_bits(want)) ++mismatches;
                }
            }
        }
    }
    printf("%lld %lld\n", checked, mismatches);
    return mismatches != 0;
}
