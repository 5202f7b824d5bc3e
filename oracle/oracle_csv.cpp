// ORACLE — test infrastructure only (see oracle.h). CPU restatement of the CLI's CSV output,
// writeCsv (src/main.zig:181-198), and of the number rendering it relies on: Zig's "{d}"
// (Zig standard library 0.17.1, lib/std/fmt/float.zig — a dependency absent from the reference
// tree). That rendering is Ryu (U. Adams, PLDI 2018): the shortest decimal digits that read back
// to the same float, the closest such string to the exact value when several have that length
// (ties to even), printed in decimal notation without an exponent.
//
// Two restatements of the f32 digits are kept: oracle_f32_digits, Ryu with 125-bit multipliers
// (the parameterisation of Zig's 64-bit backend, wider than the 59/61-bit one of the GPU kernels),
// and oracle_f32_digits_search, a plain search over digit counts with glibc's correctly rounded
// printf / strtof, used only to pin the first one.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "oracle.h"

namespace {

typedef unsigned __int128 u128;

constexpr int kInvBits = 125, kPosBits = 125;

int pow5bits(int e) { return (int)(((uint32_t)e * 1217359u) >> 19) + 1; }
uint32_t log10pow2(int e) { return ((uint32_t)e * 78913u) >> 18; }
uint32_t log10pow5(int e) { return ((uint32_t)e * 732923u) >> 20; }

// floor(2^n / d), d < 2^110, quotient < 2^126.
u128 div_pow2(int n, u128 d) {
    u128 rem = 0, q = 0;
    for (int b = n; b >= 0; --b) {
        rem = (rem << 1) | (u128)(b == n);
        q <<= 1;
        if (rem >= d) {
            rem -= d;
            q |= 1;
        }
    }
    return q;
}

struct Tables {
    u128 inv[32];  // floor(2^(pow5bits(q) - 1 + 125) / 5^q) + 1
    u128 pos[48];  // 5^i * 2^(125 - pow5bits(i))
    Tables() {
        u128 p = 1;
        for (int q = 0; q < 32; ++q, p *= 5) inv[q] = div_pow2(pow5bits(q) - 1 + kInvBits, p) + 1;
        p = 1;
        for (int i = 0; i < 48; ++i, p *= 5) pos[i] = p << (kPosBits - pow5bits(i));
    }
};

const Tables &tables() {
    static const Tables t;
    return t;
}

// (m * f) >> shift for m < 2^32, f < 2^126, 64 < shift < 158.
uint32_t mul_shift(uint32_t m, u128 f, int shift) {
    const u128 b0 = (u128)m * (uint64_t)f, b2 = (u128)m * (uint64_t)(f >> 64);
    return (uint32_t)(((b0 >> 64) + b2) >> (shift - 64));
}

int pow5_factor(uint32_t v) {
    int c = 0;
    while (v != 0 && v % 5 == 0) {
        v /= 5;
        ++c;
    }
    return c;
}

// Ryu's digit generation for a finite non-zero f32 magnitude.
void ryu_f32(uint32_t bits, uint32_t *digits, int32_t *exponent) {
    const Tables &t = tables();
    const uint32_t mant = bits & 0x7fffffu, expo = (bits >> 23) & 0xffu;
    const int e2 = (expo == 0 ? 1 : (int)expo) - 127 - 23 - 2;
    const uint32_t m2 = expo == 0 ? mant : ((1u << 23) | mant);
    const bool accept = (m2 & 1u) == 0;
    const uint32_t mv = 4 * m2, mp = mv + 2, mm_shift = (mant != 0 || expo <= 1) ? 1 : 0, mm = mv - 1 - mm_shift;
    uint32_t vr, vp, vm, last = 0;
    int e10;
    bool vr_tz = false, vm_tz = false;
    if (e2 >= 0) {
        // vr = floor(mv * 2^e2 / 10^q)
        const uint32_t q = log10pow2(e2);
        e10 = (int)q;
        const int sh = -e2 + (int)q + kInvBits + pow5bits((int)q) - 1;
        vr = mul_shift(mv, t.inv[q], sh);
        vp = mul_shift(mp, t.inv[q], sh);
        vm = mul_shift(mm, t.inv[q], sh);
        if (q != 0 && (vp - 1) / 10 <= vm / 10) {
            const int sh1 = -e2 + (int)q - 1 + kInvBits + pow5bits((int)q - 1) - 1;
            last = mul_shift(mv, t.inv[q - 1], sh1) % 10;
        }
        if (q <= 9) {
            // The removed part of vr is zero iff 5^q divides mv (2^q divides 2^e2).
            if (mv % 5 == 0) {
                vr_tz = pow5_factor(mv) >= (int)q;
            } else if (accept) {
                vm_tz = pow5_factor(mm) >= (int)q;
            } else if (pow5_factor(mp) >= (int)q) {
                --vp;
            }
        }
    } else {
        // vr = floor(mv * 5^i / 2^q), i = -e2 - q
        const uint32_t q = log10pow5(-e2);
        e10 = (int)q + e2;
        const int i = -e2 - (int)q;
        const int sh = (int)q - (pow5bits(i) - kPosBits);
        vr = mul_shift(mv, t.pos[i], sh);
        vp = mul_shift(mp, t.pos[i], sh);
        vm = mul_shift(mm, t.pos[i], sh);
        if (q != 0 && (vp - 1) / 10 <= vm / 10) {
            const int sh1 = (int)q - 1 - (pow5bits(i + 1) - kPosBits);
            last = mul_shift(mv, t.pos[i + 1], sh1) % 10;
        }
        if (q <= 1) {
            vr_tz = true;
            if (accept) {
                vm_tz = mm_shift == 1;
            } else {
                --vp;
            }
        } else if (q < 31) {
            // Digits below the last removed one are zero iff 2^(q-1) divides mv.
            vr_tz = (mv & ((1u << (q - 1)) - 1)) == 0;
        }
    }
    int removed = 0;
    uint32_t out;
    if (vm_tz || vr_tz) {
        while (vp / 10 > vm / 10) {
            vm_tz = vm_tz && vm % 10 == 0;
            vr_tz = vr_tz && last == 0;
            last = vr % 10;
            vr /= 10, vp /= 10, vm /= 10;
            ++removed;
        }
        if (vm_tz)
            while (vm % 10 == 0) {
                vr_tz = vr_tz && last == 0;
                last = vr % 10;
                vr /= 10, vp /= 10, vm /= 10;
                ++removed;
            }
        if (vr_tz && last == 5 && vr % 2 == 0) last = 4;
        out = vr + (((vr == vm && (!accept || !vm_tz)) || last >= 5) ? 1 : 0);
    } else {
        while (vp / 10 > vm / 10) {
            last = vr % 10;
            vr /= 10, vp /= 10, vm /= 10;
            ++removed;
        }
        out = vr + ((vr == vm || last >= 5) ? 1 : 0);
    }
    *digits = out;
    *exponent = e10 + removed;
}

// Decimal notation of digits * 10^exponent (formatDecimal of lib/std/fmt/float.zig).
size_t decimal_text(bool neg, const std::string &digits, int exponent, char *out) {
    std::string s = neg ? "-" : "";
    const int nd = (int)digits.size(), dp = exponent + nd;
    if (dp <= 0) {
        s += "0." + std::string(-dp, '0') + digits;
    } else if (dp >= nd) {
        s += digits + std::string(dp - nd, '0');
    } else {
        s += digits.substr(0, dp) + "." + digits.substr(dp);
    }
    std::memcpy(out, s.data(), s.size());
    return s.size();
}

// Special values as Zig prints them: "nan" (unsigned), "inf" / "-inf", "0" / "-0".
bool special_text(double x, char *out, size_t *n) {
    const char *s = nullptr;
    if (std::isnan(x)) s = "nan";
    else if (std::isinf(x)) s = x < 0 ? "-inf" : "inf";
    else if (x == 0) s = std::signbit(x) ? "-0" : "0";
    if (!s) return false;
    *n = std::strlen(s);
    std::memcpy(out, s, *n);
    return true;
}

// Shortest round-trip digits by search: for each digit count, the correctly rounded candidate,
// then its neighbour on the other side of x; the first that reads back wins.
template <class T>
void search_digits(T x, int max_len, std::string *digits, int *exponent) {
    char buf[64];
    for (int len = 1; len <= max_len; ++len) {
        snprintf(buf, sizeof buf, "%.*e", len - 1, (double)x);
        const char *e = std::strchr(buf, 'e');
        std::string d;
        for (const char *c = buf; c < e; ++c)
            if (*c >= '0' && *c <= '9') d += *c;
        const int ex = std::atoi(e + 1) - (len - 1);
        const T back = sizeof(T) == 4 ? (T)std::strtof(buf, nullptr) : (T)std::strtod(buf, nullptr);
        if (back == x) {
            *digits = d;
            *exponent = ex;
            break;
        }
        unsigned long long v = std::strtoull(d.c_str(), nullptr, 10);
        v = std::strtod(buf, nullptr) < (double)x ? v + 1 : v - 1;
        snprintf(buf, sizeof buf, "%llue%d", v, ex);
        const T back2 = sizeof(T) == 4 ? (T)std::strtof(buf, nullptr) : (T)std::strtod(buf, nullptr);
        if (v > 0 && back2 == x) {
            *digits = std::to_string(v);
            *exponent = ex;
            break;
        }
    }
    while (digits->size() > 1 && digits->back() == '0') {
        digits->pop_back();
        ++*exponent;
    }
}

size_t f32_text(float x, char *out) {
    size_t n;
    if (special_text(x, out, &n)) return n;
    uint32_t bits;
    std::memcpy(&bits, &x, 4);
    uint32_t d;
    int32_t e;
    ryu_f32(bits & 0x7fffffffu, &d, &e);
    return decimal_text(std::signbit(x), std::to_string(d), e, out);
}

size_t f64_text(double x, char *out) {
    size_t n;
    if (special_text(x, out, &n)) return n;
    std::string d;
    int e = 0;
    search_digits<double>(std::fabs(x), 17, &d, &e);
    return decimal_text(std::signbit(x), d, e, out);
}

size_t u64_text(uint64_t v, char *out) {
    char tmp[24];
    int n = 0;
    do {
        tmp[n++] = (char)('0' + v % 10);
        v /= 10;
    } while (v);
    for (int i = 0; i < n; ++i) out[i] = tmp[n - 1 - i];
    return (size_t)n;
}

// One line "s,v,step,x0,...\n" into out (at most 63 + 50 * q bytes); returns its length.
size_t line_text(const float *values, size_t line, size_t variates, size_t horizon, size_t q, char *out) {
    size_t n = 0;
    n += u64_text(line / (variates * horizon), out + n);
    out[n++] = ',';
    n += u64_text((line / horizon) % variates, out + n);
    out[n++] = ',';
    n += u64_text(line % horizon + 1, out + n);
    for (size_t j = 0; j < q; ++j) {
        out[n++] = ',';
        n += f32_text(values[line * q + j], out + n);
    }
    out[n++] = '\n';
    return n;
}

}  // namespace

extern "C" {

void oracle_f32_digits(float x, uint32_t *digits, int32_t *exponent) {
    uint32_t bits;
    std::memcpy(&bits, &x, 4);
    ryu_f32(bits & 0x7fffffffu, digits, exponent);
}

void oracle_f32_digits_search(float x, uint64_t *digits, int32_t *exponent) {
    std::string d;
    int e = 0;
    search_digits<float>(std::fabs(x), 9, &d, &e);
    *digits = std::strtoull(d.c_str(), nullptr, 10);
    *exponent = e;
}

void oracle_f32_digits_batch(const float *x, size_t n, uint32_t *digits, int32_t *exponent) {
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; ++i) oracle_f32_digits(x[i], digits + i, exponent + i);
}

void oracle_f32_digits_search_batch(const float *x, size_t n, uint64_t *digits, int32_t *exponent) {
#pragma omp parallel for schedule(dynamic, 4096)
    for (size_t i = 0; i < n; ++i) oracle_f32_digits_search(x[i], digits + i, exponent + i);
}

size_t oracle_f32_text(float x, char *out) { return f32_text(x, out); }

size_t oracle_f64_text(double x, char *out) { return f64_text(x, out); }

// writeCsv (src/main.zig:181-198) into out when capacity allows; returns the text's length.
// Lines are rendered in parallel (OpenMP) into per-thread spans, then placed in order.
size_t oracle_csv_format(const float *values, size_t series, size_t variates, size_t horizon, const double *levels,
                         size_t nq, char *out, size_t capacity) {
    std::string head = "series,variate,step";
    char tmp[64];
    for (size_t i = 0; i < nq; ++i) {
        head += ",q";
        head.append(tmp, f64_text(levels[i], tmp));
    }
    head += '\n';
    const size_t lines = series * variates * horizon;
    std::vector<uint32_t> len(lines);
#pragma omp parallel
    {
        std::vector<char> buf(64 + 50 * nq);
#pragma omp for schedule(static)
        for (size_t l = 0; l < lines; ++l) len[l] = (uint32_t)line_text(values, l, variates, horizon, nq, buf.data());
    }
    std::vector<size_t> off(lines + 1, head.size());
    for (size_t l = 0; l < lines; ++l) off[l + 1] = off[l] + len[l];
    const size_t total = off[lines];
    if (out == nullptr || total > capacity) return total;
    std::memcpy(out, head.data(), head.size());
#pragma omp parallel for schedule(static)
    for (size_t l = 0; l < lines; ++l) line_text(values, l, variates, horizon, nq, out + off[l]);
    return total;
}

}  // extern "C"
