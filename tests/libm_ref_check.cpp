// Host build of quantr-in-c_b200/csrc/libm_ref.cuh checked against the C
// library's expf over every float bit pattern (NaN results compare as NaN).
// Built and run by tests/test_libm_ref.py.  Prints "mismatches N".
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>

#include "libm_ref.cuh"

int main()
{
    unsigned long long bad = 0;
#pragma omp parallel for schedule(static) reduction(+ : bad)
    for (long long hi = 0; hi < 65536; ++hi) {
        for (uint32_t lo = 0; lo < 65536; ++lo) {
            const uint32_t u = (uint32_t)(hi << 16) | lo;
            float x;
            std::memcpy(&x, &u, 4);
            const float a = expf(x), b = qr::libm::expf_ref(x);
            uint32_t ua, ub;
            std::memcpy(&ua, &a, 4);
            std::memcpy(&ub, &b, 4);
            if (ua != ub && !(std::isnan(a) && std::isnan(b))) ++bad;
        }
    }
    std::printf("mismatches %llu\n", bad);
    return bad != 0;
}
