/* Exhaustive check used by tests/test_div127.py: the scale of a Q8_0 block,
 * d = amax / 127 (IEEE single division, round to nearest), equals
 *     q = RN(amax * r), r = RN(1/127);  e = fma(-q, 127, amax);  d' = fma(e, r, q)
 * for every non-negative finite float amax.  The device code computes d this
 * way (common.cuh div127_rn); both use only correctly rounded operations, so
 * agreement here is agreement on the GPU. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

int main(void) {
    const float r   = 1.0f / 127.0f;
    uint64_t    bad = 0;
    for (uint64_t u = 0; u < 0x7f800000ull; ++u) {
        const uint32_t bits = (uint32_t) u;
        float          a;
        memcpy(&a, &bits, 4);
        const float q   = a * r;
        const float e   = fmaf(-q, 127.0f, a);
        const float d   = fmaf(e, r, q);
        const float ref = a / 127.0f;
        if (memcmp(&d, &ref, 4) != 0) {
            ++bad;
        }
    }
    printf("%llu\n", (unsigned long long) bad);
    return bad != 0;
}
