/* Host model of div127 (fl_common.cuh): q0 = RN(y * RN(1/127)),
 * e = fma(-q0, 127, y), q = copysign(fma(e, RN(1/127), q0), y), compared
 * bit for bit with the correctly rounded y / 127 for every float whose
 * biased exponent is in the ranges given as arguments (pairs lo hi), both
 * signs. Prints "tested N bad M"; exit status 1 on any mismatch. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

int main(int argc, char** argv) {
    const float b = 127.0f;
    volatile float one = 1.0f;
    const float r = one / b;
    unsigned long long tested = 0, bad = 0;
    for (int a = 1; a + 1 < argc; a += 2) {
        const uint32_t lo = (uint32_t)atoi(argv[a]), hi = (uint32_t)atoi(argv[a + 1]);
        for (uint32_t ex = lo; ex <= hi && ex < 255; ex++)
            for (uint32_t sign = 0; sign < 2; sign++)
                for (uint32_t man = 0; man < (1u << 23); man++) {
                    const uint32_t w = (sign << 31) | (ex << 23) | man;
                    float y;
                    memcpy(&y, &w, 4);
                    const float want = y / b;
                    const float q0 = y * r;
                    const float e = fmaf(-q0, b, y);
                    const float q = copysignf(fmaf(e, r, q0), y);
                    uint32_t x0, x1;
                    memcpy(&x0, &want, 4);
                    memcpy(&x1, &q, 4);
                    tested++;
                    if (x0 != x1) {
                        if (bad < 5) printf("mismatch %a: %a against %a\n", y, q, want);
                        bad++;
                    }
                }
    }
    printf("tested %llu bad %llu\n", tested, bad);
    return bad != 0;
}
