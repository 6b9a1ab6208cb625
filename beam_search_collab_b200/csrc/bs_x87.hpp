// bs_x87.hpp -- arithmetic at the precision of the x87 extended format.
//
// The reference codebook builder computes two of its three per-edge factors
// in `long double` (src/build_rabitq.cpp:247-252):
//   x_x0      = (long double)r_norm / fac_x0
//   triple_x  = (float)((long double)r_norm * r_norm + 2.0L * x_x0 * fac_x1)
//   factor_dq = (float)(-2.0L * x_x0 * fac_norm)
// On x86-64 Linux `long double` is the 80-bit x87 format with precision
// control at 64 bits: every operation rounds its exact result to a 64-bit
// significand (round to nearest, ties to even), and the final conversion
// rounds that again to float.  The GPU has no such format, so this header
// carries the few operations those formulas need, in integer arithmetic with
// the same roundings: a value is m * 2^(e-63) with bit 63 of m set.  NaNs
// produced by invalid operations are the x87 default NaN (negative, quiet),
// which converts to the float 0xffc00000.
//
// Host and device code share it (a host test compares it against the
// compiler's own long double).
#pragma once

#include <cstdint>
#include <cstring>

#if defined(__CUDACC__)
#define BS_X87_FN __host__ __device__ __forceinline__
#else
#define BS_X87_FN inline
#endif

namespace bsb {
namespace x87 {

enum : uint32_t { kZero = 0, kFinite = 1, kInf = 2, kNan = 3 };

struct Xf {
    uint64_t m;     // significand (bit 63 set when finite), NaN payload
    int32_t e;      // value = m * 2^(e - 63)
    uint32_t neg;   // sign bit
    uint32_t cls;   // kZero / kFinite / kInf / kNan
};

BS_X87_FN int clz64(uint64_t x) {
#if defined(__CUDA_ARCH__)
    return __clzll(static_cast<long long>(x));
#else
    return x ? __builtin_clzll(x) : 64;
#endif
}

BS_X87_FN void mul64x64(uint64_t a, uint64_t b, uint64_t& hi, uint64_t& lo) {
#if defined(__CUDA_ARCH__)
    lo = a * b;
    hi = __umul64hi(a, b);
#else
    const unsigned __int128 p = static_cast<unsigned __int128>(a) * b;
    lo = static_cast<uint64_t>(p);
    hi = static_cast<uint64_t>(p >> 64);
#endif
}

BS_X87_FN Xf make(uint64_t m, int32_t e, uint32_t neg, uint32_t cls) {
    Xf x;
    x.m = m;
    x.e = e;
    x.neg = neg;
    x.cls = cls;
    return x;
}

BS_X87_FN Xf default_nan() { return make(0xc000000000000000ull, 0, 1u, kNan); }

BS_X87_FN Xf from_float(float f) {
    uint32_t b;
    std::memcpy(&b, &f, 4);
    const uint32_t neg = b >> 31, ex = (b >> 23) & 0xffu, fr = b & 0x7fffffu;
    if (ex == 0xffu) {
        if (fr == 0) return make(0x8000000000000000ull, 0, neg, kInf);
        // quiet NaN with the float's payload
        return make(0xc000000000000000ull | (static_cast<uint64_t>(fr) << 40), 0, neg, kNan);
    }
    if (ex == 0) {
        if (fr == 0) return make(0, 0, neg, kZero);
        const uint64_t m = static_cast<uint64_t>(fr);   // subnormal: fr * 2^-149
        const int lz = clz64(m);
        return make(m << lz, -149 + 63 - lz, neg, kFinite);
    }
    return make((static_cast<uint64_t>(fr) | 0x800000ull) << 40, static_cast<int32_t>(ex) - 127, neg, kFinite);
}

// (hi:lo) has bit 127 set; value = (hi:lo) * 2^(e - 127).  Rounds to a 64-bit
// significand, ties to even; `sticky` = nonzero bits below lo.
BS_X87_FN Xf round128(uint64_t hi, uint64_t lo, int32_t e, bool sticky, uint32_t neg) {
    const bool rbit = (lo >> 63) != 0;
    const bool rest = sticky || (lo << 1) != 0;
    uint64_t m = hi;
    if (rbit && (rest || (m & 1u))) {
        ++m;
        if (m == 0) {
            m = 0x8000000000000000ull;
            ++e;
        }
    }
    return make(m, e, neg, kFinite);
}

BS_X87_FN Xf mul(const Xf& a, const Xf& b) {
    const uint32_t neg = a.neg ^ b.neg;
    if (a.cls == kNan) return a;
    if (b.cls == kNan) return b;
    if (a.cls == kInf || b.cls == kInf) {
        if (a.cls == kZero || b.cls == kZero) return default_nan();
        return make(0x8000000000000000ull, 0, neg, kInf);
    }
    if (a.cls == kZero || b.cls == kZero) return make(0, 0, neg, kZero);
    uint64_t hi, lo;
    mul64x64(a.m, b.m, hi, lo);   // in [2^126, 2^128)
    int32_t e = a.e + b.e + 1;
    if (!(hi >> 63)) {
        hi = (hi << 1) | (lo >> 63);
        lo <<= 1;
        e -= 1;
    }
    return round128(hi, lo, e, false, neg);
}

// a / b for operands that are floats (24-bit significands), by long division.
BS_X87_FN Xf div_floats(const Xf& a, const Xf& b) {
    const uint32_t neg = a.neg ^ b.neg;
    if (a.cls == kNan) return a;
    if (b.cls == kNan) return b;
    if (a.cls == kInf) {
        if (b.cls == kInf) return default_nan();
        return make(0x8000000000000000ull, 0, neg, kInf);
    }
    if (b.cls == kInf) return make(0, 0, neg, kZero);
    if (b.cls == kZero) {
        if (a.cls == kZero) return default_nan();
        return make(0x8000000000000000ull, 0, neg, kInf);   // divide by zero, masked
    }
    if (a.cls == kZero) return make(0, 0, neg, kZero);
    uint64_t ma = a.m >> 40, mb = b.m >> 40;   // 24-bit significands
    int32_t e = a.e - b.e;
    if (ma < mb) {
        ma <<= 1;
        e -= 1;
    }
    uint64_t q = 0, rem = ma;
    for (int i = 0; i < 64; ++i) {
        const bool bit = rem >= mb;
        if (bit) rem -= mb;
        q = (q << 1) | (bit ? 1u : 0u);
        rem <<= 1;
    }
    const bool rbit = rem >= mb;
    if (rbit) rem -= mb;
    const bool sticky = rem != 0;
    if (rbit && (sticky || (q & 1u))) {
        ++q;
        if (q == 0) {
            q = 0x8000000000000000ull;
            ++e;
        }
    }
    return make(q, e, neg, kFinite);
}

BS_X87_FN Xf add(const Xf& a0, const Xf& b0) {
    if (a0.cls == kNan) return a0;
    if (b0.cls == kNan) return b0;
    if (a0.cls == kInf || b0.cls == kInf) {
        if (a0.cls == kInf && b0.cls == kInf && a0.neg != b0.neg) return default_nan();
        return a0.cls == kInf ? a0 : b0;
    }
    if (a0.cls == kZero && b0.cls == kZero) return make(0, 0, a0.neg & b0.neg, kZero);
    if (a0.cls == kZero) return b0;
    if (b0.cls == kZero) return a0;
    // |a| >= |b|
    const bool swap = (b0.e > a0.e) || (b0.e == a0.e && b0.m > a0.m);
    const Xf& a = swap ? b0 : a0;
    const Xf& b = swap ? a0 : b0;
    const int32_t diff = a.e - b.e;
    if (diff >= 66) return a;   // |b| below half an ulp of a: the sum rounds to a
    // a at bits 62..125 of a 128-bit window, b shifted right by diff below it
    const uint64_t ahi = a.m >> 2, alo = a.m << 62;
    uint64_t bhi = b.m >> 2, blo = b.m << 62;
    bool lost = false;
    if (diff >= 64) {
        const int s = diff - 64;
        lost = s > 0 && (bhi << (64 - s)) != 0;
        lost = lost || blo != 0;
        blo = s ? (bhi >> s) : bhi;
        bhi = 0;
    } else if (diff > 0) {
        lost = (blo << (64 - diff)) != 0;
        blo = (blo >> diff) | (bhi << (64 - diff));
        bhi >>= diff;
    }
    uint64_t shi, slo;
    if (a.neg == b.neg) {
        slo = alo + blo;
        shi = ahi + bhi + (slo < alo ? 1u : 0u);
    } else {
        slo = alo - blo;
        shi = ahi - bhi - (alo < blo ? 1u : 0u);
        if (lost) {
            // the exact difference lies strictly between S - 1 and S
            shi -= (slo == 0 ? 1u : 0u);
            slo -= 1u;
        }
        if (shi == 0 && slo == 0 && !lost) return make(0, 0, 0u, kZero);
    }
    int lz = shi ? clz64(shi) : 64 + clz64(slo);
    if (lz >= 64) {
        shi = slo;
        slo = 0;
        lz -= 64;
    }
    if (lz > 0) {
        shi = (shi << lz) | (slo >> (64 - lz));
        slo <<= lz;
    }
    // bit 125 of the window stood for 2^(a.e); after the shift bit 127 is the leading one
    return round128(shi, slo, a.e + 2 - lz, lost, a.neg);
}

// Conversion to float, rounding to nearest, ties to even (subnormals and
// overflow as IEEE).
BS_X87_FN float to_float(const Xf& x) {
    uint32_t b;
    if (x.cls == kNan) {
        b = (x.neg << 31) | 0x7fc00000u | static_cast<uint32_t>((x.m >> 40) & 0x7fffffu);
    } else if (x.cls == kInf) {
        b = (x.neg << 31) | 0x7f800000u;
    } else if (x.cls == kZero) {
        b = x.neg << 31;
    } else {
        int32_t e = x.e;
        int sh = 40;                       // keep 24 bits
        if (e < -126) sh += -126 - e;      // subnormal result
        uint64_t keep = 0;
        bool rbit = false, sticky = false;
        if (sh >= 65) {
            keep = 0;
            rbit = false;
            sticky = true;
        } else {
            keep = sh < 64 ? (x.m >> sh) : 0;
            rbit = ((x.m >> (sh - 1)) & 1u) != 0;
            sticky = sh > 1 && (x.m & ((1ull << (sh - 1)) - 1u)) != 0;
        }
        if (rbit && (sticky || (keep & 1u))) ++keep;
        if (e < -126) {
            b = (x.neg << 31) | static_cast<uint32_t>(keep);   // 0x800000 = smallest normal
        } else {
            if (keep == (1ull << 24)) {
                keep >>= 1;
                ++e;
            }
            if (e > 127) b = (x.neg << 31) | 0x7f800000u;
            else b = (x.neg << 31) | (static_cast<uint32_t>(e + 127) << 23) | static_cast<uint32_t>(keep & 0x7fffffu);
        }
    }
    float f;
    std::memcpy(&f, &b, 4);
    return f;
}

// The reference builder's two long-double factors of one edge
// (src/build_rabitq.cpp:247-252), from its float inputs.
BS_X87_FN void edge_factors(float r_norm, float fac_x0, float fac_x1, float fac_norm, float& triple_x,
                            float& factor_dq) {
    const Xf r = from_float(r_norm);
    const Xf x_x0 = div_floats(r, from_float(fac_x0));
    const Xf t = add(mul(r, r), mul(mul(from_float(2.0f), x_x0), from_float(fac_x1)));
    triple_x = to_float(t);
    factor_dq = to_float(mul(mul(from_float(-2.0f), x_x0), from_float(fac_norm)));
}

}  // namespace x87
}  // namespace bsb
