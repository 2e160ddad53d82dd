// x86_numerics.h -- host side of the reference-exact numerics mode (see exact_math.cuh).
//
// The reference's compiled decode engine runs three operations whose results are not fixed by
// IEEE 754: the RSQRTSS and RCPPS estimates (Newton-refined by GCC under -ffast-math) and the C
// library's expf.  This file captures them from the host the library runs on -- the machine the
// reference runs on -- as tables the GPU evaluates exactly:
//   * RCPSS / RSQRTSS: 2048 outputs each, then a check that the table model (top mantissa bits,
//     exact exponent scaling, flush of tiny results) reproduces the instruction on every mantissa
//     of a binade and on sampled inputs of every exponent;
//   * expf: every float x in [-112, -0] whose expf(x) differs from exp((double)x) rounded to float,
//     or whose double result lies within 1e-6 ulp of a rounding midpoint (there another double exp
//     could round the other way), as sorted (x bits, expf bits) pairs.  ~1.1e9 inputs, split over
//     all host threads; built once per process.
// Host code only (compiled in the host pass of asdsl_b200.cu).
#pragma once

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "exact_math.cuh"

#if defined(__x86_64__) || defined(__i386__)
#define ASDSL_HOST_X86 1
#if !defined(__CUDA_ARCH__)
#include <xmmintrin.h>
#endif
#endif

namespace asdsl {

struct HostExactTables {
    uint32_t rcp[kRcpTabSize];
    uint32_t rsqrt[kRsqrtTabSize];
    std::vector<uint32_t> exp_exc;  // pairs (x bits, expf bits), x bits ascending
    bool ok = false;
    std::string err;
};

inline uint32_t host_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}
inline float host_float(uint32_t u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

#ifdef ASDSL_HOST_X86
// (the device compilation pass parses these host functions too; it never runs them)
#if !defined(__CUDA_ARCH__)
inline uint32_t host_rcpss(uint32_t x) { return host_bits(_mm_cvtss_f32(_mm_rcp_ss(_mm_set_ss(host_float(x))))); }
inline uint32_t host_rsqrtss(uint32_t x) {
    return host_bits(_mm_cvtss_f32(_mm_rsqrt_ss(_mm_set_ss(host_float(x)))));
}
#else
inline uint32_t host_rcpss(uint32_t) { return 0; }
inline uint32_t host_rsqrtss(uint32_t) { return 0; }
#endif

// 1/sqrt(a) as GCC -ffast-math emits it (RSQRTSS + one Newton step), on this host
inline float host_nr_rsqrt(float a) {
    const float x0 = host_float(host_rsqrtss(host_bits(a)));
    const float t = std::fma(x0, x0 * a, -3.0f);
    return t * (x0 * -0.5f);
}

inline void build_exp_exceptions(std::vector<uint32_t>& out) {
    const uint32_t lo = 0x80000000u, hi = 0xC2E00000u;  // -0 .. -112 (expf underflows below ~-103.97)
    unsigned nt = std::thread::hardware_concurrency();
    if (nt == 0) nt = 4;
    if (nt > 64) nt = 64;
    std::vector<std::vector<uint32_t>> part(nt);
    std::vector<std::thread> th;
    const uint64_t span = static_cast<uint64_t>(hi) - lo + 1;
    for (unsigned t = 0; t < nt; ++t) {
        th.emplace_back([&, t]() {
            const uint64_t a = lo + span * t / nt, b = lo + span * (t + 1) / nt;
            std::vector<uint32_t>& v = part[t];
            for (uint64_t u = a; u < b; ++u) {
                const float x = host_float(static_cast<uint32_t>(u));
                const float f = expf(x);
                const double y = std::exp(static_cast<double>(x));
                const float g = static_cast<float>(y);
                bool keep = host_bits(f) != host_bits(g);
                if (!keep && g >= 1.17549435e-38f) {
                    const double gd = g;
                    const double up = host_float(host_bits(g) + 1u), dn = host_float(host_bits(g) - 1u);
                    const double dup = ((gd + up) * 0.5 - y) / (up - gd);
                    const double ddn = (y - (gd + dn) * 0.5) / (gd - dn);
                    keep = dup < 1e-6 || ddn < 1e-6;
                }
                if (keep) {
                    v.push_back(static_cast<uint32_t>(u));
                    v.push_back(host_bits(f));
                }
            }
        });
    }
    for (auto& x : th) x.join();
    out.clear();
    for (auto& v : part) out.insert(out.end(), v.begin(), v.end());  // threads cover ascending ranges
}

inline bool build_host_exact_tables(HostExactTables& T) {
    for (int i = 0; i < kRcpTabSize; ++i) T.rcp[i] = host_rcpss(0x3F800000u | (static_cast<uint32_t>(i) << 12));
    for (int i = 0; i < kRsqrtTabSize; ++i) {
        const uint32_t e = 127u + static_cast<uint32_t>(i >> 10);
        T.rsqrt[i] = host_rsqrtss((e << 23) | (static_cast<uint32_t>(i & 1023) << 13));
    }
    // the table model must reproduce the instruction: every mantissa of [1,2) (and [2,4) for
    // RSQRTSS), and sampled mantissas of every normal exponent, both signs for RCPSS
    for (uint32_t m = 0; m < (1u << 23); ++m) {
        const uint32_t x = 0x3F800000u | m, x2 = 0x40000000u | m;
        if (emu_rcp_bits(x, T.rcp) != host_rcpss(x) || emu_rsqrt_bits(x, T.rsqrt) != host_rsqrtss(x) ||
            emu_rsqrt_bits(x2, T.rsqrt) != host_rsqrtss(x2)) {
            T.err = "host RCPSS/RSQRTSS do not follow the table model (mantissa " + std::to_string(m) + ")";
            return false;
        }
    }
    for (uint32_t e = 1; e < 255; ++e)
        for (uint32_t m = 0; m < (1u << 23); m += 4093) {
            const uint32_t x = (e << 23) | m;
            if (emu_rcp_bits(x, T.rcp) != host_rcpss(x) || emu_rcp_bits(x | 0x80000000u, T.rcp) != host_rcpss(x | 0x80000000u) ||
                emu_rsqrt_bits(x, T.rsqrt) != host_rsqrtss(x)) {
                T.err = "host RCPSS/RSQRTSS do not follow the table model (exponent " + std::to_string(e) + ")";
                return false;
            }
        }
    build_exp_exceptions(T.exp_exc);
    T.ok = true;
    return true;
}
#endif  // ASDSL_HOST_X86

// the process-wide tables (built on first use; an error string when the host cannot supply them)
inline const HostExactTables& host_exact_tables() {
    static HostExactTables T;
    static std::once_flag once;
    std::call_once(once, []() {
#ifdef ASDSL_HOST_X86
        build_host_exact_tables(T);
#else
        T.err = "the reference-exact numerics mode needs an x86 host (RCPSS/RSQRTSS/expf of the reference's CPU)";
#endif
    });
    return T;
}

}  // namespace asdsl
