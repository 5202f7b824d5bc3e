// Decimal / hexadecimal text to f64, correctly rounded (round half to even), for the series
// reader (core/series.zig:15-19: `std.fmt.parseFloat(f64, s) catch nan`). Accepted: an optional
// sign, then a decimal number (digits with an optional point and an optional e/E exponent), a
// hexadecimal number (0x / 0X, hex digits with an optional point and an optional p/P binary
// exponent), or inf / infinity / nan in any case; anything else is not a number (NaN). Host and
// device share this header.
//
// Paths, fastest first, all exact:
//   (1) at most 15 significant digits and a decimal exponent in [-22, 22]: one IEEE multiply or
//       divide of two exactly representable doubles (Clinger);
//   (2) at most 19 significant digits and an exponent in [-19, 19]: the value as a 128-bit
//       integer (w * 10^e) or a 128-by-64-bit quotient (w * 2^s / 10^m) with a sticky remainder,
//       rounded once;
//   (3) otherwise: up to 800 significant digits in a multi-word integer (more are folded into a
//       sticky flag: 800 decimal digits decide the rounding of every double), times 10^e or
//       divided by 10^m with a 65-bit quotient by shift-and-subtract, rounded once.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define TSFM_PHD __host__ __device__ __forceinline__
#define TSFM_PHD_NOINLINE __host__ __device__ __noinline__
#else
#define TSFM_PHD inline
#define TSFM_PHD_NOINLINE inline
#endif

namespace tsfm {
namespace numparse {

typedef unsigned __int128 u128;

TSFM_PHD double bits_to_double(uint64_t b) {
    union {
        uint64_t u;
        double d;
    } x;
    x.u = b;
    return x.d;
}

TSFM_PHD double quiet_nan(bool neg) { return bits_to_double((neg ? 0x8000000000000000ull : 0) | 0x7ff8000000000000ull); }
TSFM_PHD double infinity(bool neg) { return bits_to_double((neg ? 0x8000000000000000ull : 0) | 0x7ff0000000000000ull); }

TSFM_PHD int clz64(uint64_t x) {
#if defined(__CUDA_ARCH__)
    return __clzll((long long)x);
#else
    return x ? __builtin_clzll(x) : 64;
#endif
}

TSFM_PHD int bitlen128(u128 x) {
    const uint64_t hi = (uint64_t)(x >> 64);
    return hi ? 128 - clz64(hi) : 64 - clz64((uint64_t)x);
}

// Rounds (q + frac) * 2^b to a double, where q > 0 and `sticky` says whether frac > 0;
// frac < 1 is only known through the sticky flag, so q must carry at least 2 bits beyond the
// 53 kept (the rounding bit and one more) whenever the result is normal.
TSFM_PHD double round_scaled(u128 q, int b, bool sticky, bool neg) {
    const int n = bitlen128(q);
    int e = b + n - 1;  // exponent of the leading bit
    if (e > 1023) return infinity(neg);
    // Bits of q below the last kept one: 53 kept for normals, fewer for subnormals.
    int keep = 53;
    if (e < -1022) keep = 53 - (-1022 - e);
    const int drop = n - keep;
    uint64_t m;
    if (keep <= 0) {
        // Below half the smallest subnormal, or exactly at / above it (keep == 0: q's leading bit
        // is the rounding bit of 2^-1074).
        if (keep < 0) return bits_to_double(neg ? 0x8000000000000000ull : 0);
        const bool above = (q & ((((u128)1) << (n - 1)) - 1)) != 0 || sticky;
        m = above ? 1 : 0;  // exactly half rounds to even (0)
        return bits_to_double((neg ? 0x8000000000000000ull : 0) | m);
    }
    if (drop <= 0) {
        m = (uint64_t)(q << (-drop));  // callers pass a q with spare bits whenever sticky is set
    } else {
        m = (uint64_t)(q >> drop);
        const u128 rem = q & ((((u128)1) << drop) - 1), half = ((u128)1) << (drop - 1);
        if (rem > half || (rem == half && (sticky || (m & 1)))) ++m;
    }
    // m has `keep` bits (or keep + 1 after a carry).
    uint64_t bits;
    if (e < -1022) {
        if (m >> keep) {  // carried into the next binade
            ++e;
        }
        bits = m;  // subnormal (or the smallest normal after a carry: m == 2^52 sets the exponent bit)
    } else {
        if (m >> 53) {
            m >>= 1;
            ++e;
            if (e > 1023) return infinity(neg);
        }
        bits = ((uint64_t)(e + 1023) << 52) | (m & ((1ull << 52) - 1));
    }
    return bits_to_double((neg ? 0x8000000000000000ull : 0) | bits);
}

// ----- path (3): multi-word integers, 32-bit limbs, least significant first -----
constexpr int kMaxDigits = 800;
constexpr int kLimbs = 136;  // 10^1150 < 2^3821 < 2^(32 * 120); room for shifts

struct Big {
    int n;  // limbs in use
    uint32_t w[kLimbs];
};

TSFM_PHD void big_set(Big &a, uint32_t v) {
    a.n = v ? 1 : 0;
    a.w[0] = v;
}
TSFM_PHD void big_mul_small(Big &a, uint32_t m, uint32_t add) {
    uint64_t carry = add;
    for (int i = 0; i < a.n; ++i) {
        const uint64_t t = (uint64_t)a.w[i] * m + carry;
        a.w[i] = (uint32_t)t;
        carry = t >> 32;
    }
    if (carry && a.n < kLimbs) a.w[a.n++] = (uint32_t)carry;
}
TSFM_PHD int big_bits(const Big &a) {
    if (a.n == 0) return 0;
    const uint32_t top = a.w[a.n - 1];
    return 32 * (a.n - 1) + (32 - clz64((uint64_t)top) + 32);
}
// a <<= s
TSFM_PHD void big_shl(Big &a, int s) {
    if (a.n == 0 || s == 0) return;
    const int ws = s / 32, bs = s % 32;
    int n = a.n + ws + 1;
    if (n > kLimbs) n = kLimbs;
    for (int i = n - 1; i >= 0; --i) {
        const int src = i - ws;
        uint32_t v = 0;
        if (src >= 0 && src < a.n) v = a.w[src] << bs;
        if (bs && src - 1 >= 0 && src - 1 < a.n) v |= a.w[src - 1] >> (32 - bs);
        a.w[i] = v;
    }
    a.n = n;
    while (a.n > 0 && a.w[a.n - 1] == 0) --a.n;
}
TSFM_PHD int big_cmp(const Big &a, const Big &b) {
    if (a.n != b.n) return a.n < b.n ? -1 : 1;
    for (int i = a.n - 1; i >= 0; --i)
        if (a.w[i] != b.w[i]) return a.w[i] < b.w[i] ? -1 : 1;
    return 0;
}
// a -= b (a >= b)
TSFM_PHD void big_sub(Big &a, const Big &b) {
    int64_t borrow = 0;
    for (int i = 0; i < a.n; ++i) {
        int64_t t = (int64_t)a.w[i] - (i < b.n ? (int64_t)b.w[i] : 0) - borrow;
        borrow = t < 0;
        a.w[i] = (uint32_t)(t + (borrow << 32));
    }
    while (a.n > 0 && a.w[a.n - 1] == 0) --a.n;
}
TSFM_PHD void big_shr1(Big &a) {
    for (int i = 0; i < a.n; ++i) a.w[i] = (a.w[i] >> 1) | (i + 1 < a.n ? a.w[i + 1] << 31 : 0);
    while (a.n > 0 && a.w[a.n - 1] == 0) --a.n;
}
TSFM_PHD void big_pow10(Big &a, int e) {  // a *= 10^e
    while (e >= 9) {
        big_mul_small(a, 1000000000u, 0);
        e -= 9;
    }
    uint32_t p = 1;
    while (e-- > 0) p *= 10;
    if (p > 1) big_mul_small(a, p, 0);
}

// Exact value of digits[0..nd) (most significant first) * 10^e10, truncated digits flagged by
// `more`, rounded to a double.
TSFM_PHD_NOINLINE double slow_path(const uint8_t *digits, int nd, int e10, bool more, bool neg) {
    Big num, den;
    big_set(num, 0);
    for (int i = 0; i < nd; ++i) big_mul_small(num, 10, digits[i]);
    if (num.n == 0) return bits_to_double(neg ? 0x8000000000000000ull : 0);
    if (e10 >= 0) {
        big_pow10(num, e10);
        const int n = big_bits(num);
        // Top 64 bits with a sticky flag for the rest.
        u128 q = 0;
        bool sticky = more;
        const int lo = n > 64 ? n - 64 : 0;
        for (int bit = n - 1; bit >= lo; --bit) q = (q << 1) | ((num.w[bit / 32] >> (bit % 32)) & 1);
        for (int bit = 0; bit < lo && !sticky; ++bit) sticky = ((num.w[bit / 32] >> (bit % 32)) & 1) != 0;
        return round_scaled(q, lo, sticky, neg);
    }
    // num / 10^m: scale so the quotient has 65 bits, then shift-and-subtract.
    big_set(den, 1);
    big_pow10(den, -e10);
    const int s = 65 + big_bits(den) - big_bits(num);
    if (s > 0) {
        big_shl(num, s);
    } else if (s < 0) {
        big_shl(den, -s);
    }
    // Now num / den < 2^66.
    Big sh = den;
    big_shl(sh, 65);
    u128 q = 0;
    for (int k = 65; k >= 0; --k) {
        q <<= 1;
        if (big_cmp(num, sh) >= 0) {
            big_sub(num, sh);
            q |= 1;
        }
        big_shr1(sh);
    }
    return round_scaled(q, -s, num.n != 0 || more, neg);
}

TSFM_PHD bool is_digit(char c) { return c >= '0' && c <= '9'; }
TSFM_PHD int hex_value(char c) {
    if (c >= '0' && c <= '9') return c - '0';
    if (c >= 'a' && c <= 'f') return c - 'a' + 10;
    if (c >= 'A' && c <= 'F') return c - 'A' + 10;
    return -1;
}
TSFM_PHD char lower(char c) { return (c >= 'A' && c <= 'Z') ? (char)(c + 32) : c; }
TSFM_PHD bool equals_ci(const char *p, int n, const char *word) {
    int i = 0;
    for (; word[i]; ++i)
        if (i >= n || lower(p[i]) != word[i]) return false;
    return i == n;
}

// 10^e for 0 <= e <= 22: every partial product is an integer below 2^53 times a power of two,
// so each multiplication is exact.
TSFM_PHD double pow10_exact(int e) {
    double p = 1.0;
    while (e-- > 0) p *= 10.0;
    return p;
}

TSFM_PHD uint64_t pow10_u64(int e) {
    uint64_t p = 1;
    while (e-- > 0) p *= 10;
    return p;
}

// Hexadecimal significand (after "0x") with an optional binary exponent; exact to 64 bits plus a
// sticky flag for further non-zero digits.
TSFM_PHD double parse_hex(const char *p, int n, bool neg, bool *ok) {
    u128 m = 0;
    int shift = 0;  // binary exponent contributed by dropped or fractional digits
    bool sticky = false, any = false, point = false;
    int i = 0;
    for (; i < n; ++i) {
        const char c = p[i];
        if (c == '.') {
            if (point) break;
            point = true;
            continue;
        }
        const int v = hex_value(c);
        if (v < 0) break;
        any = true;
        if ((m >> 60) == 0) {
            m = (m << 4) | (u128)v;
            if (point) shift -= 4;
        } else {
            sticky |= v != 0;
            if (!point) shift += 4;
        }
    }
    if (!any) {
        *ok = false;
        return 0;
    }
    if (i < n && (p[i] == 'p' || p[i] == 'P')) {
        ++i;
        bool eneg = false;
        if (i < n && (p[i] == '+' || p[i] == '-')) eneg = p[i++] == '-';
        if (i >= n || !is_digit(p[i])) {
            *ok = false;
            return 0;
        }
        int ex = 0;
        for (; i < n && is_digit(p[i]); ++i)
            if (ex < 100000) ex = ex * 10 + (p[i] - '0');
        shift += eneg ? -ex : ex;
    }
    if (i != n) {
        *ok = false;
        return 0;
    }
    *ok = true;
    if (m == 0) return bits_to_double(neg ? 0x8000000000000000ull : 0);
    // Keep at least 2 bits of room below the 53 kept for round_scaled's rounding bit.
    return round_scaled(m, shift, sticky, neg);
}

// High 128 bits of the 256-bit product a * b.
TSFM_PHD u128 mulhi128(u128 a, u128 b) {
    const uint64_t a0 = (uint64_t)a, a1 = (uint64_t)(a >> 64), b0 = (uint64_t)b, b1 = (uint64_t)(b >> 64);
    const u128 p00 = (u128)a0 * b0, p01 = (u128)a0 * b1, p10 = (u128)a1 * b0, p11 = (u128)a1 * b1;
    const u128 mid = (p00 >> 64) + (uint64_t)p01 + (uint64_t)p10;  // < 3 * 2^64
    return p11 + (p01 >> 64) + (p10 >> 64) + (mid >> 64);
}

// floor(2^128 / 10^m) for m in [1, 19] (index m), the reciprocals of path (2): the quotient
// estimate mulhi(num, r) is at most 2 below the true quotient and is corrected exactly.
struct Recip10 {
    u128 r[20];
};

inline Recip10 make_recip10() {
    Recip10 t{};
    u128 d = 1;
    for (int m = 1; m < 20; ++m) {
        d *= 10;
        t.r[m] = (~(u128)0) / d;  // floor((2^128 - 1) / d) == floor(2^128 / d) for d not a power of 2
    }
    return t;
}

// Parses the whole of p[0, n) (already trimmed); NaN when it is not a number. `recip`, when
// given, replaces the 128-bit division of path (2) by a multiply and at most two corrections.
TSFM_PHD_NOINLINE double parse_number(const char *p, int n, const Recip10 *recip = nullptr) {
    int i = 0;
    bool neg = false;
    if (i < n && (p[i] == '+' || p[i] == '-')) neg = p[i++] == '-';
    if (i >= n) return quiet_nan(false);
    const char c0 = lower(p[i]);
    if (c0 == 'i' || c0 == 'n') {
        if (equals_ci(p + i, n - i, "inf") || equals_ci(p + i, n - i, "infinity")) return infinity(neg);
        if (equals_ci(p + i, n - i, "nan")) return quiet_nan(neg);
        return quiet_nan(false);
    }
    if (p[i] == '0' && i + 1 < n && (p[i + 1] == 'x' || p[i + 1] == 'X')) {
        bool ok = false;
        const double v = parse_hex(p + i + 2, n - i - 2, neg, &ok);
        return ok ? v : quiet_nan(false);
    }
    // Decimal: significant digits (leading zeros skipped), the point's position, the exponent.
    uint64_t w = 0;
    int nsig = 0, dropped = 0, frac = 0;
    bool any = false, point = false, more = false;
    const int start = i;
    for (; i < n; ++i) {
        const char c = p[i];
        if (c == '.') {
            if (point) break;
            point = true;
            continue;
        }
        if (!is_digit(c)) break;
        any = true;
        const int d = c - '0';
        if (point) ++frac;
        if (nsig == 0 && d == 0) continue;
        if (nsig < 19) {
            w = w * 10 + (uint64_t)d;
            ++nsig;
        } else {
            ++dropped;
            more |= d != 0;
        }
    }
    const int mant_end = i;
    if (!any) return quiet_nan(false);
    int ex = 0;
    if (i < n && (p[i] == 'e' || p[i] == 'E')) {
        ++i;
        bool eneg = false;
        if (i < n && (p[i] == '+' || p[i] == '-')) eneg = p[i++] == '-';
        if (i >= n || !is_digit(p[i])) return quiet_nan(false);
        for (; i < n && is_digit(p[i]); ++i)
            if (ex < 100000) ex = ex * 10 + (p[i] - '0');
        if (eneg) ex = -ex;
    }
    if (i != n) return quiet_nan(false);
    if (w == 0) return bits_to_double(neg ? 0x8000000000000000ull : 0);
    // value = w * 10^e10 (+ dropped digits)
    const int e10 = ex + dropped - frac;
    if (!more) {  // dropped digits, if any, are zeros: w * 10^e10 is exact
        if (w <= (1ull << 53) && e10 >= -22 && e10 <= 22) {
            const double x = (double)w;
            const double v = e10 >= 0 ? x * pow10_exact(e10) : x / pow10_exact(-e10);
            return neg ? -v : v;
        }
        if (e10 >= 0 && e10 <= 19) return round_scaled((u128)w * pow10_u64(e10), 0, false, neg);
        if (e10 < 0 && e10 >= -19) {
            const int s = 127 - bitlen128((u128)w);
            const u128 num = ((u128)w) << s;
            const uint64_t den = pow10_u64(-e10);
            u128 q, rem;
            if (recip != nullptr) {
                q = mulhi128(num, recip->r[-e10]);
                rem = num - q * den;
                while (rem >= den) {
                    rem -= den;
                    ++q;
                }
            } else {
                q = num / den;
                rem = num - q * den;
            }
            return round_scaled(q, -s, rem != 0, neg);
        }
    }
    // Path (3): gather up to kMaxDigits significant digits again.
    uint8_t digits[kMaxDigits];
    int nd = 0, pos_frac = 0;
    bool started = false, seen_point = false, tail = false;
    for (int k = start; k < mant_end; ++k) {
        const char c = p[k];
        if (c == '.') {
            seen_point = true;
            continue;
        }
        const int d = c - '0';
        if (seen_point) ++pos_frac;
        if (!started && d == 0) continue;
        started = true;
        if (nd < kMaxDigits) {
            digits[nd++] = (uint8_t)d;
        } else {
            tail |= d != 0;
            if (seen_point) --pos_frac;  // a dropped fractional digit does not move the point
            else ++ex;                   // a dropped integer digit scales by 10
        }
    }
    const int e = ex - pos_frac;
    // Far outside the double range: no need for the multi-word arithmetic.
    if (e + nd > 310) return infinity(neg);
    if (e + nd < -330) return bits_to_double(neg ? 0x8000000000000000ull : 0);
    return slow_path(digits, nd, e, tail, neg);
}

}  // namespace numparse
}  // namespace tsfm
