// exact_math.cuh -- the reference-exact numerics mode: the fp32 operations the reference's
// compiled CPU code performs, reproduced on the GPU bit for bit.
//
// The reference is built with g++ -O3 -ffast-math (setup.py:56-65).  Under that flag GCC emits,
// for the decode engine (asdsl/kernels/native/unified_engine.cpp):
//   * `1.0f / std::sqrt(a)` (rmsnorm_f32 :499-524, residual_add_rmsnorm_f32 :663-693, attention's
//     1/sqrt(head_dim) :924) as RSQRTSS plus one Newton step: t = fma(x0, x0*a, -3), r = t*(x0*-0.5);
//   * the vector divide of swiglu_inplace's sigmoid (:845) as RCPPS plus one Newton step:
//     r = (x0 + x0) - x0*(x0*d);
//   * attention's std::exp (:989, :1000) as a call to the C library's expf.
// RSQRTSS/RCPPS are table-driven approximations whose exact outputs depend on the CPU (they are
// not IEEE operations).  On the host they depend only on the top 10 (RSQRTSS, plus the exponent
// parity) or 11 (RCPPS) mantissa bits of the input and scale exactly with its exponent; the host
// captures the 2048-entry tables from its own CPU and verifies that model over a full binade and
// every exponent (x86_numerics.h), and the GPU evaluates the same model here.  expf is computed
// as exp() in double rounded to float -- the correctly rounded result -- except where the C
// library's expf rounds the other way; the host enumerates those inputs over the whole domain the
// attention uses (every float <= 0 down to full underflow) into a sorted table, and the GPU looks
// an input up only when its double result lies within 1/100 ulp of a float rounding midpoint
// (the C library's misrounded inputs all lie within 2e-3 ulp of one).
#pragma once

#include <cstdint>

namespace asdsl {

constexpr int kRcpTabSize = 2048;    // RCPPS: top 11 mantissa bits
constexpr int kRsqrtTabSize = 2048;  // RSQRTSS: exponent parity x top 10 mantissa bits

// Device copies of the host tables (one set per device, filled once).
struct ExactTabs {
    const uint32_t* rcp;      // [2048] RCPSS output bits for inputs 1 + i/2048 (exponent 127)
    const uint32_t* rsqrt;    // [2048] RSQRTSS output bits: [0,1024) inputs in [1,2), [1024,2048) in [2,4)
    // the expf exceptions as an open-addressing hash table: slots of (input bits, libm expf
    // output bits), empty slots keyed kExpHashEmpty, linear probing from exp_hash_slot(key)
    const uint2* exp_hash;
    uint32_t exp_hash_mask;   // slots - 1 (a power of two)
    int exp_hash_shift;       // 32 - log2(slots)
    int n_exp_exc;            // exceptions listed
};

constexpr uint32_t kExpHashEmpty = 0xFFFFFFFFu;  // a NaN pattern: never an input of the attention's expf

__host__ __device__ __forceinline__ uint32_t exp_hash_slot(uint32_t key, int shift) {
    return (key * 0x9E3779B1u) >> shift;  // multiplicative hashing spreads runs of adjacent keys
}

// RCPSS on a positive or negative normal input: the table entry of its mantissa, its exponent
// moved by the input's; results below the normal range are flushed to a signed zero (as the
// instruction does), zeros and denormals give a signed infinity.
__host__ __device__ __forceinline__ uint32_t emu_rcp_bits(uint32_t x, const uint32_t* tab) {
    const uint32_t sign = x & 0x80000000u;
    const int e = static_cast<int>((x >> 23) & 0xFFu);
    if (e == 0) return sign | 0x7F800000u;
    if (e == 255) return (x & 0x7FFFFFu) ? x : sign;  // NaN stays NaN, 1/inf = 0
    const uint32_t t = tab[(x >> 12) & 0x7FFu];
    const int re = static_cast<int>((t >> 23) & 0xFFu) - (e - 127);
    if (re <= 0) return sign;
    if (re >= 255) return sign | 0x7F800000u;
    return sign | (static_cast<uint32_t>(re) << 23) | (t & 0x7FFFFFu);
}

// RSQRTSS on a positive normal input (the only inputs it gets here: sum/n + eps, head_dim).
__host__ __device__ __forceinline__ uint32_t emu_rsqrt_bits(uint32_t x, const uint32_t* tab) {
    const int e = static_cast<int>((x >> 23) & 0xFFu);
    const int par = (e - 127) & 1;           // exponent parity: [1,2) or [2,4) binade pair
    const int k = (e - 127 - par) / 2;       // exact: even numerator
    const uint32_t t = tab[par * 1024 + ((x >> 13) & 0x3FFu)];
    const int re = static_cast<int>((t >> 23) & 0xFFu) - k;
    return (static_cast<uint32_t>(re) << 23) | (t & 0x7FFFFFu);
}

#ifdef __CUDACC__
// GCC -ffast-math's 1/sqrt(a): RSQRTSS estimate + one Newton step, operand order as emitted
__device__ __forceinline__ float exact_nr_rsqrt(float a, const uint32_t* tab) {
    const float x0 = __uint_as_float(emu_rsqrt_bits(__float_as_uint(a), tab));
    const float t = __fmaf_rn(x0, __fmul_rn(x0, a), -3.0f);
    return __fmul_rn(t, __fmul_rn(x0, -0.5f));
}

// GCC -ffast-math's 1/d for a vector divide: RCPPS estimate + one Newton step
__device__ __forceinline__ float exact_nr_recip(float d, const uint32_t* tab) {
    const float x0 = __uint_as_float(emu_rcp_bits(__float_as_uint(d), tab));
    const float e = __fmul_rn(x0, __fmul_rn(x0, d));
    return __fsub_rn(__fadd_rn(x0, x0), e);
}

// swiglu_inplace's vector body (unified_engine.cpp:836-857 with fast_exp_avx2 :803-825 inlined),
// in the compiled order: 1 + p*2^i is one FMA, sigmoid = 1/d by RCPPS + Newton, val = (g*u)*sigmoid.
__device__ __forceinline__ float exact_silu_mul(float g, float u, const uint32_t* rcp_tab) {
    float x = -g;
    x = fmaxf(x, -87.3f);
    x = fminf(x, 87.3f);
    x = __fmul_rn(x, 1.4426950408889634f);
    const int i = __float2int_rn(x);
    const float f = __fsub_rn(x, static_cast<float>(i));
    float p = __fmaf_rn(0.001333838100523091f, f, 0.009618129107628477f);
    p = __fmaf_rn(p, f, 0.05550410866482158f);
    p = __fmaf_rn(p, f, 0.2402265069591007f);
    p = __fmaf_rn(p, f, 0.6931471805599453f);
    p = __fmaf_rn(p, f, 1.0f);
    const float d = __fmaf_rn(p, __int_as_float((i + 127) << 23), 1.0f);
    return __fmul_rn(__fmul_rn(g, u), exact_nr_recip(d, rcp_tab));
}

// The C library's expf on x <= 0: exp in double, rounded to float; near a rounding midpoint (or
// for results below the normal range) the host-enumerated exception table decides.
__device__ __forceinline__ float exact_expf(float x, const ExactTabs& t) {
    const double y = exp(static_cast<double>(x));
    const float f = __double2float_rn(y);
    bool hard = !(f >= 1.17549435e-38f);  // zero or subnormal result
    if (!hard) {
        const double fd = static_cast<double>(f);
        const double up = static_cast<double>(__uint_as_float(__float_as_uint(f) + 1u));
        const double dn = static_cast<double>(__uint_as_float(__float_as_uint(f) - 1u));
        // within 1/100 of the spacing of a rounding midpoint on either side (the spacings are
        // positive: compared by multiplication, no double division)
        hard = (((fd + up) * 0.5 - y) < 0.01 * (up - fd)) || ((y - (fd + dn) * 0.5) < 0.01 * (fd - dn));
    }
    if (hard) {
        // the table is at most a quarter full, so a probe run ends at an empty slot within a slot
        // or two (one cache line); the loop bound only guards a malformed table
        const uint32_t key = __float_as_uint(x);
        uint32_t i = exp_hash_slot(key, t.exp_hash_shift);
        for (uint32_t probe = 0; probe <= t.exp_hash_mask; ++probe) {
            const uint2 e = __ldg(t.exp_hash + i);
            if (e.x == key) return __uint_as_float(e.y);
            if (e.x == kExpHashEmpty) break;
            i = (i + 1u) & t.exp_hash_mask;
        }
    }
    return f;
}
#endif  // __CUDACC__

}  // namespace asdsl
