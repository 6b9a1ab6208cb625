// Test program: the x87-precision emulation of bs_x87.hpp against the host
// compiler's own long double (x86-64: 80-bit x87, 64-bit significand) on the
// reference builder's two factor formulas (src/build_rabitq.cpp:247-252).
// Prints "<differing> <checked>" and exits 1 on any difference.
#include <cfloat>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>

#include "bs_x87.hpp"

static unsigned bits_of(float f) {
    unsigned b;
    std::memcpy(&b, &f, 4);
    return b;
}

int main(int argc, char** argv) {
    const long per = argc > 1 ? std::atol(argv[1]) : 200000;
    std::mt19937_64 g(20261202);
    long bad = 0, n = 0;
    auto check = [&](float r, float f0, float f1, float fn) {
        const long double x_x0 = static_cast<long double>(r) / f0;
        const float t = static_cast<float>(static_cast<long double>(r) * r + 2.0L * x_x0 * f1);
        const float dq = static_cast<float>(-2.0L * x_x0 * fn);
        float t2, dq2;
        bsb::x87::edge_factors(r, f0, f1, fn, t2, dq2);
        ++n;
        if (bits_of(t) != bits_of(t2) || bits_of(dq) != bits_of(dq2)) {
            if (bad < 5)
                std::printf("r=%a f0=%a f1=%a fn=%a: %08x %08x vs %08x %08x\n", r, f0, f1, fn, bits_of(t),
                            bits_of(dq), bits_of(t2), bits_of(dq2));
            ++bad;
        }
    };
    std::uniform_real_distribution<float> sym(-1.0f, 1.0f), pos(1e-3f, 2.0f);
    std::uniform_int_distribution<unsigned> any;
    // the builder's value ranges
    for (long i = 0; i < per; ++i) check(pos(g), pos(g), sym(g), 1.0f / std::sqrt(96.0f));
    // arbitrary bit patterns: zeros, subnormals, infinities, huge and tiny
    for (long i = 0; i < per; ++i) {
        float v[4];
        bool nan = false;
        for (float& x : v) {
            const unsigned b = any(g);
            std::memcpy(&x, &b, 4);
            nan = nan || std::isnan(x);
        }
        if (!nan) check(std::fabs(v[0]), v[1], v[2], v[3]);
    }
    // near-cancellation of r*r against 2*x_x0*fac_x1
    for (long i = 0; i < per; ++i) {
        const float r = pos(g), f0 = pos(g);
        const long double x = static_cast<long double>(r) / f0;
        float f1 = static_cast<float>(-static_cast<long double>(r) * r / (2.0L * x));
        f1 = std::nextafter(f1, (i & 1) ? 1.0f : -1.0f);
        check(r, f0, f1, pos(g));
    }
    // duplicate rows (fac_x0 = 0), overflow and underflow of the float result
    check(1.0f, 0.0f, 0.0f, 0.1f);
    check(1.0f, 0.0f, 1.0f, 0.1f);
    check(1e-10f, 0.0f, -3.0f, 0.1f);
    check(1.0f, 1.0f, -0.5f, 0.1f);
    check(3.0f, 1e-30f, 1e30f, 1e-30f);
    check(1e30f, 1e-30f, 1e30f, 1e30f);
    check(1e-20f, 1e20f, 1e-20f, 1e-20f);
    std::printf("%ld %ld\n", bad, n);
    return bad != 0;
}
