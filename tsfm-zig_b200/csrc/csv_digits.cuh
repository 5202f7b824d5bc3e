// Text rendering of forecast numbers as the reference CLI prints them (src/main.zig:181-198,
// `out.print("{d}", ...)`): integers in decimal; f32 values in decimal notation (no exponent)
// with the shortest digit string that reads back to the same f32, ties between two shortest
// candidates going to the one closer to the exact value (then to the even digit). The digits
// come from Ryu (U. Adams, "Ryu: fast float-to-string conversion", PLDI 2018), the algorithm
// behind Zig's std.fmt float rendering: the rounding interval of the value is scaled by a
// 59/61-bit approximation of 5^-q or 5^i, and decimal digits are removed while the interval's
// bounds still differ. Host and device share this header.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define TSFM_HD __host__ __device__ __forceinline__
#else
#define TSFM_HD inline
#endif

namespace tsfm {
namespace csv {

constexpr int kPow5InvBits = 59;   // bit width of the ceil(2^k / 5^q) multipliers
constexpr int kPow5Bits = 61;      // bit width of the floor(5^i / 2^k) multipliers
constexpr int kPow5InvCount = 32;  // q in [0, 31]: e2 >= 0 needs q <= log10(2^102) = 30
constexpr int kPow5Count = 48;     // i in [0, 47]: e2 < 0 needs i <= 46 (+1 for the removed digit)

// Multiplier tables, built on the host with exact integer arithmetic (csv.cu).
struct Pow5Tables {
    uint64_t inv[kPow5InvCount];  // floor(2^(pow5bits(q) - 1 + 59) / 5^q) + 1
    uint64_t pos[kPow5Count];     // floor(5^i / 2^(pow5bits(i) - 61)) (or 5^i * 2^(61 - pow5bits(i)))
};

// ceil(log2(5^e)) for e >= 1, and 1 for e = 0 (valid for e < 3529).
TSFM_HD int pow5bits(int e) { return (int)(((uint32_t)e * 1217359u) >> 19) + 1; }
// floor(e * log10(2)) for 0 <= e <= 1650; floor(e * log10(5)) for 0 <= e <= 2620.
TSFM_HD uint32_t log10_pow2(int e) { return ((uint32_t)e * 78913u) >> 18; }
TSFM_HD uint32_t log10_pow5(int e) { return ((uint32_t)e * 732923u) >> 20; }

TSFM_HD bool multiple_of_pow5(uint32_t v, uint32_t p) {
    uint32_t c = 0;
    while (v != 0 && v % 5 == 0) {
        v /= 5;
        ++c;
    }
    return c >= p;
}
TSFM_HD bool multiple_of_pow2(uint32_t v, uint32_t p) { return (v & ((1u << p) - 1)) == 0; }

// (m * f) >> shift for m < 2^26, f < 2^61 and 32 < shift < 96: exact 96-bit product.
TSFM_HD uint32_t mul_shift(uint32_t m, uint64_t f, int shift) {
    const uint64_t lo = (uint64_t)m * (uint32_t)f, hi = (uint64_t)m * (f >> 32);
    return (uint32_t)(((lo >> 32) + hi) >> (shift - 32));
}

// value = digits * 10^exponent, digits without trailing zeros beyond what the value needs.
struct Decimal {
    uint32_t digits;
    int32_t exponent;
};

// Shortest round-trip digits of a finite, non-zero f32 given by its bits (sign ignored).
TSFM_HD Decimal shortest(uint32_t bits, const Pow5Tables &t) {
    const uint32_t mant = bits & 0x7fffffu, expo = (bits >> 23) & 0xffu;
    int e2;
    uint32_t m2;
    if (expo == 0) {
        e2 = 1 - 127 - 23 - 2;
        m2 = mant;
    } else {
        e2 = (int)expo - 127 - 23 - 2;
        m2 = (1u << 23) | mant;
    }
    // Bounds of the rounding interval, scaled by 4: [mm, mp] around mv. Both bounds read back
    // to this value (round-half-even) exactly when its significand is even.
    const bool accept = (m2 & 1u) == 0;
    const uint32_t mv = 4 * m2, mp = 4 * m2 + 2;
    const uint32_t mm_shift = (mant != 0 || expo <= 1) ? 1u : 0u;  // the lower gap halves at 2^k
    const uint32_t mm = 4 * m2 - 1 - mm_shift;

    uint32_t vr, vp, vm, last = 0;
    int e10;
    bool vm_tz = false, vr_tz = false;
    if (e2 >= 0) {
        const uint32_t q = log10_pow2(e2);
        e10 = (int)q;
        const int k = kPow5InvBits + pow5bits((int)q) - 1;
        const int i = -e2 + (int)q + k;
        vr = mul_shift(mv, t.inv[q], i);
        vp = mul_shift(mp, t.inv[q], i);
        vm = mul_shift(mm, t.inv[q], i);
        if (q != 0 && (vp - 1) / 10 <= vm / 10) {
            // At most one digit is removed below: that digit decides the rounding.
            const int l = kPow5InvBits + pow5bits((int)q - 1) - 1;
            last = mul_shift(mv, t.inv[q - 1], -e2 + (int)q - 1 + l) % 10;
        }
        if (q <= 9) {
            // Only one of mv, mp, mm can be a multiple of 5.
            if (mv % 5 == 0) {
                vr_tz = multiple_of_pow5(mv, q);
            } else if (accept) {
                vm_tz = multiple_of_pow5(mm, q);
            } else {
                vp -= multiple_of_pow5(mp, q) ? 1u : 0u;
            }
        }
    } else {
        const uint32_t q = log10_pow5(-e2);
        e10 = (int)q + e2;
        const int i = -e2 - (int)q;
        const int k = pow5bits(i) - kPow5Bits;
        int j = (int)q - k;
        vr = mul_shift(mv, t.pos[i], j);
        vp = mul_shift(mp, t.pos[i], j);
        vm = mul_shift(mm, t.pos[i], j);
        if (q != 0 && (vp - 1) / 10 <= vm / 10) {
            j = (int)q - 1 - (pow5bits(i + 1) - kPow5Bits);
            last = mul_shift(mv, t.pos[i + 1], j) % 10;
        }
        if (q <= 1) {
            // mv = 4 * m2 has two trailing zero bits, mp one, mm one exactly when mm_shift is 1.
            vr_tz = true;
            if (accept) {
                vm_tz = mm_shift == 1;
            } else {
                --vp;
            }
        } else if (q < 31) {
            vr_tz = multiple_of_pow2(mv, q - 1);
        }
    }

    // Remove digits while the interval's bounds differ in the remaining digits.
    int removed = 0;
    uint32_t out;
    if (vm_tz || vr_tz) {
        while (vp / 10 > vm / 10) {
            vm_tz &= vm % 10 == 0;
            vr_tz &= last == 0;
            last = vr % 10;
            vr /= 10;
            vp /= 10;
            vm /= 10;
            ++removed;
        }
        if (vm_tz) {
            while (vm % 10 == 0) {
                vr_tz &= last == 0;
                last = vr % 10;
                vr /= 10;
                vp /= 10;
                vm /= 10;
                ++removed;
            }
        }
        if (vr_tz && last == 5 && vr % 2 == 0) last = 4;  // exact tie: round half to even
        out = vr + (((vr == vm && (!accept || !vm_tz)) || last >= 5) ? 1u : 0u);
    } else {
        while (vp / 10 > vm / 10) {
            last = vr % 10;
            vr /= 10;
            vp /= 10;
            vm /= 10;
            ++removed;
        }
        out = vr + ((vr == vm || last >= 5) ? 1u : 0u);
    }
    return Decimal{out, e10 + removed};
}

TSFM_HD int decimal_length(uint32_t v) {
    int n = 1;
    while (v >= 10) {
        v /= 10;
        ++n;
    }
    return n;
}

// A formatted f32: sign, kind and digits; `len` is the byte count of its text.
struct F32Text {
    uint32_t digits;
    int32_t exponent;
    int16_t len;
    int8_t ndigits;
    int8_t kind;  // 0 finite non-zero, 1 zero, 2 inf, 3 nan
    bool neg;
};

TSFM_HD F32Text describe(uint32_t bits, const Pow5Tables &t) {
    F32Text f{};
    f.neg = (bits >> 31) != 0;
    const uint32_t mag = bits & 0x7fffffffu;
    if (mag == 0) {
        f.kind = 1;
        f.len = (int16_t)(1 + f.neg);  // "0" / "-0"
    } else if (mag == 0x7f800000u) {
        f.kind = 2;
        f.len = (int16_t)(3 + f.neg);  // "inf" / "-inf"
    } else if (mag > 0x7f800000u) {
        f.kind = 3;
        f.neg = false;
        f.len = 3;  // "nan", never signed
    } else {
        const Decimal d = shortest(mag, t);
        f.digits = d.digits;
        f.exponent = d.exponent;
        f.ndigits = (int8_t)decimal_length(d.digits);
        const int dp = d.exponent + f.ndigits;
        int n;
        if (dp <= 0) {
            n = 2 - dp + f.ndigits;  // 0.000ddd
        } else if (dp >= f.ndigits) {
            n = dp;                  // ddd000
        } else {
            n = f.ndigits + 1;       // dd.ddd
        }
        f.len = (int16_t)(n + f.neg);
    }
    return f;
}

// Writes the text of `f` at p (f.len bytes).
TSFM_HD void emit(const F32Text &f, char *p) {
    if (f.neg) *p++ = '-';
    if (f.kind == 1) {
        *p = '0';
        return;
    }
    if (f.kind == 2) {
        p[0] = 'i', p[1] = 'n', p[2] = 'f';
        return;
    }
    if (f.kind == 3) {
        p[0] = 'n', p[1] = 'a', p[2] = 'n';
        return;
    }
    const int nd = f.ndigits, dp = f.exponent + nd;
    // Digits are written from the least significant one straight to their places.
    uint32_t v = f.digits;
    if (dp <= 0) {  // 0.000ddd
        p[0] = '0';
        p[1] = '.';
        for (int i = 0; i < -dp; ++i) p[2 + i] = '0';
        char *d = p + 2 - dp;
        for (int i = nd - 1; i >= 0; --i) {
            d[i] = (char)('0' + v % 10);
            v /= 10;
        }
    } else if (dp >= nd) {  // ddd000
        for (int i = nd - 1; i >= 0; --i) {
            p[i] = (char)('0' + v % 10);
            v /= 10;
        }
        for (int i = nd; i < dp; ++i) p[i] = '0';
    } else {  // dd.ddd
        for (int i = nd - 1; i >= dp; --i) {
            p[i + 1] = (char)('0' + v % 10);
            v /= 10;
        }
        p[dp] = '.';
        for (int i = dp - 1; i >= 0; --i) {
            p[i] = (char)('0' + v % 10);
            v /= 10;
        }
    }
}

// Writes the `len` decimal digits of v at p (len = its digit count).
TSFM_HD void emit_u64(uint64_t v, int len, char *p) {
    for (int i = len - 1; i >= 0; --i) {
        p[i] = (char)('0' + v % 10);
        v /= 10;
    }
}

}  // namespace csv
}  // namespace tsfm
