// common.cuh -- device helpers shared by every sm_100a kernel of asdsl-b200.
//
//  * bulk-copy (TMA 1-D, cp.async.bulk) + mbarrier wrappers, never multicast;
//  * bounded mbarrier waits: a wait that runs past kWaitLimitNs sets a bit in
//    the device status word and returns false, so a broken pipeline ends with
//    an error the host can read instead of hanging the GPU;
//  * the reference's A8 activation rounding, pinned to what the reference's
//    compiled code computes (asdsl/kernels/native/gemv_q4_preq_restored.cpp:505-549
//    built with -ffast-math: scale = amax * fl(1/127), inv = 127/amax IEEE,
//    q = round-to-nearest-even(x * inv) saturated to int8).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace asdsl {

// Status bits written by kernels (read and cleared by asdsl_b200_device_status).
enum : unsigned int {
    kStatusWaitFull = 1u,     // consumer gave up waiting for a stage to fill
    kStatusWaitEmpty = 2u,    // producer gave up waiting for a stage to drain
    kStatusWaitDrain = 4u,    // producer gave up draining its copies at exit
    kStatusBadLaunch = 8u,    // kernel saw an inconsistent launch configuration
    kStatusXchgWait = 16u,    // a cross-GPU exchange gave up waiting for a peer's word
};

// Wall-clock limit of any single device-side wait.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

// system-scope 64-bit store / load for words exchanged with peer GPUs over NVLink
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// relaxed system-scope forms: for words that carry their own step tag, so that no fence has to
// order other data before them (a system-scope release costs microseconds)
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// The suspend-time hint lets a waiting thread sleep (up to the hint) until the
// phase completes instead of spinning, so idle warps do not steal issue slots.
constexpr uint32_t kTryWaitSuspendNs = 100000;

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kTryWaitSuspendNs)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and the caller records a
// status bit) if the phase did not complete within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes).
// Both addresses 16-byte aligned and bytes a multiple of 16 (checked by callers).
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Same, with an L2 evict-first policy: streamed weights are read once per call.
__device__ __forceinline__ void bulk_g2s_stream(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar,
                                                uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Programmatic dependent launch: wait for the producing grid's memory to be visible
// (no-op when the kernel was not launched with the programmatic attribute).
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Numerics
// ---------------------------------------------------------------------------

// fl(1/127) and fl(1/7): the constants GCC folds `x / 127.0f`, `x / 7.0f` into
// under the reference's -ffast-math build (pinned against the compiled reference).
__device__ __forceinline__ float inv127f() { return __int_as_float(0x3c010204); }
__device__ __forceinline__ float inv7f() { return __int_as_float(0x3e124925); }

__device__ __forceinline__ float half_bits_to_float(uint32_t h16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h16 & 0xFFFFu)));
}

// both fp16 halves of a 32-bit word (low half -> .x) in one packed conversion
__device__ __forceinline__ float2 half2_bits_to_float2(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// exact float of a 4-bit code (low nibble of v) without the conversion unit
__device__ __forceinline__ float nibble_to_float(uint32_t v) {
    return __fsub_rn(__uint_as_float(0x4B000000u | (v & 0xFu)), 8388608.0f);
}

// exact int -> float for |v| < 2^22 without the conversion unit: the integer is placed in the
// mantissa of 1.5 * 2^23 and the offset subtracted (the W4A8 group dots are below 2^16)
__device__ __forceinline__ float small_int_to_float(int v) {
    return __fsub_rn(__int_as_float(0x4B400000 + v), 12582912.0f);
}

// A8 code of one value given inv = 127/amax: RNE, saturated like _mm_packs.
__device__ __forceinline__ int a8_code(float x, float inv) {
    int q = __float2int_rn(__fmul_rn(x, inv));
    q = q > 127 ? 127 : q;
    q = q < -128 ? -128 : q;
    return q;
}

// Byte offset of element j (0..31) of a 32-group inside our permuted x8 record:
// words [e0 o0 e1 o1 e2 o2 e3 o3], e_k = x[8k], x[8k+2], x[8k+4], x[8k+6] and
// o_k = x[8k+1], x[8k+3], ...  This pairs each 32-bit word of 8 packed nibbles
// (low nibbles = even elements, high = odd) with one even and one odd word.
__device__ __forceinline__ int x8_perm_offset(int j) {
    const int k = j >> 3, m = j & 7;
    return ((2 * k + (m & 1)) << 2) + (m >> 1);
}

// Integer dot of one 16-byte nibble chunk (32 weights, low nibble = even
// element) with a permuted 32-element x8 record held as two uint4.
__device__ __forceinline__ int dot_nib32(uint4 w, uint4 xa, uint4 xb, int acc) {
    const uint32_t m = 0x0F0F0F0Fu;
    acc = __dp4a(static_cast<int>(w.x & m), static_cast<int>(xa.x), acc);
    acc = __dp4a(static_cast<int>((w.x >> 4) & m), static_cast<int>(xa.y), acc);
    acc = __dp4a(static_cast<int>(w.y & m), static_cast<int>(xa.z), acc);
    acc = __dp4a(static_cast<int>((w.y >> 4) & m), static_cast<int>(xa.w), acc);
    acc = __dp4a(static_cast<int>(w.z & m), static_cast<int>(xb.x), acc);
    acc = __dp4a(static_cast<int>((w.z >> 4) & m), static_cast<int>(xb.y), acc);
    acc = __dp4a(static_cast<int>(w.w & m), static_cast<int>(xb.z), acc);
    acc = __dp4a(static_cast<int>((w.w >> 4) & m), static_cast<int>(xb.w), acc);
    return acc;
}

// 16-byte load from shared memory at a 2-byte aligned address (Q4_128 blocks
// are 66 bytes, so their nibble runs are only 2-byte aligned).  Reads up to 3
// bytes past the 16; stage buffers carry slack for that.
__device__ __forceinline__ uint4 lds128_a2(const uint8_t* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
    const uint32_t sh = static_cast<uint32_t>(a & 3u) * 8u;
    const uint32_t w0 = w[0], w1 = w[1], w2 = w[2], w3 = w[3], w4 = w[4];
    return make_uint4(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh), __funnelshift_r(w2, w3, sh),
                      __funnelshift_r(w3, w4, sh));
}

// explicit shared-memory loads on 32-bit shared-window addresses
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ float ldsf(uint32_t a) { return __uint_as_float(lds32(a)); }
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ float2 lds64f(uint32_t a) {
    const uint2 v = lds64(a);
    return make_float2(__uint_as_float(v.x), __uint_as_float(v.y));
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds8(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u8 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
// 16 bytes at a 2-byte aligned shared address (Q4_128's 66-byte blocks)
__device__ __forceinline__ uint4 lds128_a2s(uint32_t a) {
    const uint32_t b = a & ~3u, sh = (a & 3u) * 8u;
    const uint32_t w0 = lds32(b), w1 = lds32(b + 4), w2 = lds32(b + 8), w3 = lds32(b + 12), w4 = lds32(b + 16);
    return make_uint4(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh), __funnelshift_r(w2, w3, sh),
                      __funnelshift_r(w3, w4, sh));
}

// unsigned-bytes x signed-bytes dot, accumulated (dp4a.u32.s32)
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Integer dot of a 16-byte nibble run (32 weights, low nibble = even element)
// with a permuted 32-element x8 record: low nibbles in place against the even
// words, high nibbles masked in place (16x their value) against the odd words,
// combined exactly at the end.
__device__ __forceinline__ int dot_nib32_split(uint4 w, uint4 xa, uint4 xb) {
    const uint32_t lo = 0x0F0F0F0Fu, hi = 0xF0F0F0F0u;
    int dl = dp4a_us(w.x & lo, xa.x, 0);
    int dh = dp4a_us(w.x & hi, xa.y, 0);
    dl = dp4a_us(w.y & lo, xa.z, dl);
    dh = dp4a_us(w.y & hi, xa.w, dh);
    dl = dp4a_us(w.z & lo, xb.x, dl);
    dh = dp4a_us(w.z & hi, xb.y, dh);
    dl = dp4a_us(w.w & lo, xb.z, dl);
    dh = dp4a_us(w.w & hi, xb.w, dh);
    return dl + (dh >> 4);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace asdsl
