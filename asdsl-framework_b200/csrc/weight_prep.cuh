// weight_prep.cuh -- the reference's offline weight preparation, on the device.
//
// Byte-exact restatements of the NumPy pipeline that turns fp32 projection weights into the
// decode GEMVs' formats (seconds per tensor in NumPy; milliseconds here):
//   quantize_weights (clip search)   asdsl/quantization/core.py:358-424, :291-355, :57-60
//   preq blocks (scale, zero)        asdsl/quantization/repack_q4_32.py:63-102
//   preq2 split (meta + 4-row bands) asdsl/quantization/repack_preq2.py:22-46
//   Q4_128 from fp32                 asdsl/quantization/repack_q4_128.py:22-31, :72-92
//   C0.1 g128 requant source         experiments/phi4_cpu_run.py:3432-3448, :3482-3517
// Every float32 step is the reference's NumPy operation in the same order, with explicit
// round-to-nearest intrinsics so that nothing is contracted into an FMA; float64 steps stay
// float64; fp16 conversions round to nearest even, as NumPy's astype does.  The MSE of the clip
// search is summed in NumPy's float32 order for a contiguous row of n <= 128 elements (eight
// running partial sums over i, i + 8, ..., then ((r0+r1)+(r2+r3)) + ((r4+r5)+(r6+r7))).
#pragma once

#include "common.cuh"

namespace asdsl {

// clip ratios of the MSE search, as float32 (core.py:57-60)
__device__ __constant__ float kClipRatios[9] = {0.85f, 0.90f, 0.93f, 0.95f, 0.97f, 0.98f, 0.99f, 0.995f, 1.0f};

__device__ __forceinline__ float f16_round_trip(float x) { return __half2float(__float2half_rn(x)); }

__device__ __forceinline__ uint16_t f16_bits(float x) { return __half_as_ushort(__float2half_rn(x)); }

__device__ __forceinline__ uint16_t f16_bits_from_double(double x) { return __half_as_ushort(__double2half(x)); }

__device__ __forceinline__ float clampf(float v, float lo, float hi) { return fminf(fmaxf(v, lo), hi); }

// element i of group `grp` of the flattened weights, zero past numel (the reference pads the
// flattened tensor to a multiple of the group size with zeros)
template <int GS>
__device__ __forceinline__ float group_elem(const float* __restrict__ w, long long numel, long long grp, int i) {
    const long long idx = grp * GS + i;
    return idx < numel ? __ldg(w + idx) : 0.0f;
}

// float32 sum of GS values in NumPy's pairwise order (GS a multiple of 8, <= 128)
struct PairwiseSum8 {
    float r[8];
    __device__ __forceinline__ void add(int i, float v) {
        if (i < 8) r[i] = v;
        else r[i & 7] = __fadd_rn(r[i & 7], v);
    }
    __device__ __forceinline__ float total() const {
        return __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                         __fadd_rn(__fadd_rn(r[4], r[5]), __fadd_rn(r[6], r[7])));
    }
};

// One group per thread: fp16 scale (and zero), 4-bit codes packed two per byte (low nibble =
// even element).  SYM: symmetric (offset 7.5); SEARCH: MSE-optimal clip ratio.
template <int GS, bool SYM, bool SEARCH>
__global__ void k_quantize_groups(const float* __restrict__ w, long long numel, long long n_groups,
                                  uint8_t* __restrict__ packed, uint16_t* __restrict__ scales,
                                  uint16_t* __restrict__ zeros) {
    const long long grp = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (grp >= n_groups) return;
    constexpr float kQmax = 15.0f;
    float wmin = INFINITY, wmax = -INFINITY, amax = 0.0f;
#pragma unroll 8
    for (int i = 0; i < GS; ++i) {
        const float v = group_elem<GS>(w, numel, grp, i);
        wmin = fminf(wmin, v);
        wmax = fmaxf(wmax, v);
        amax = fmaxf(amax, fabsf(v));
    }
    float best_s = 0.0f, best_z = 0.0f;
    if constexpr (!SEARCH) {
        // compute_scale_zero (core.py:63-94)
        if constexpr (SYM) {
            best_s = __fdiv_rn(fmaxf(amax, 1e-5f), 7.5f);
        } else {
            const float range = fmaxf(__fsub_rn(wmax, wmin), 1e-5f);
            best_s = __fdiv_rn(range, kQmax);
            best_z = __fdiv_rn(-wmin, best_s);
        }
    } else {
        float best_mse = 0.0f;
        for (int ri = 0; ri < 9; ++ri) {
            const float r = kClipRatios[ri];
            float sc, zr = 0.0f, s16, z16;
            if constexpr (SYM) {
                // abs_max * r / (qmax / 2), floored at 1e-5 (core.py:124-129)
                sc = fmaxf(__fdiv_rn(__fmul_rn(fmaxf(amax, 1e-5f), r), 7.5f), 1e-5f);
                s16 = fmaxf(f16_round_trip(sc), 1e-4f);
                z16 = 7.5f;
            } else {
                // clipped min/max range (core.py:130-139)
                const float range = fmaxf(__fsub_rn(wmax, wmin), 1e-5f);
                const float margin = __fdiv_rn(__fmul_rn(range, __fsub_rn(1.0f, r)), 2.0f);
                const float lo = __fadd_rn(wmin, margin);
                const float hi = __fsub_rn(wmax, margin);
                const float span = fmaxf(__fsub_rn(hi, lo), 1e-5f);
                sc = __fdiv_rn(span, kQmax);
                zr = clampf(__fdiv_rn(-lo, fmaxf(sc, 1e-5f)), 0.0f, kQmax);
                s16 = fmaxf(f16_round_trip(sc), 1e-4f);
                z16 = f16_round_trip(zr);
            }
            PairwiseSum8 acc;
#pragma unroll 8
            for (int i = 0; i < GS; ++i) {
                const float v = group_elem<GS>(w, numel, grp, i);
                const float q = clampf(rintf(__fadd_rn(__fdiv_rn(v, s16), z16)), 0.0f, kQmax);
                const float d = __fsub_rn(v, __fmul_rn(__fsub_rn(q, z16), s16));
                acc.add(i, __fmul_rn(d, d));
            }
            const float mse = __fdiv_rn(acc.total(), static_cast<float>(GS));
            // first ratio with the smallest MSE (np.argmin)
            if (ri == 0 || mse < best_mse) {
                best_mse = mse;
                best_s = sc;
                best_z = zr;
            }
        }
    }
    const uint16_t sb = f16_bits(best_s);
    scales[grp] = sb;
    const float sf = fmaxf(__half2float(__ushort_as_half(sb)), 1e-4f);
    float zf = 7.5f;
    if constexpr (!SYM) {
        const uint16_t zb = f16_bits(best_z);
        zeros[grp] = zb;
        zf = __half2float(__ushort_as_half(zb));
    }
    // codes (core.py:404-413) packed as core.py:555-561, four bytes per store
    uint32_t* out = reinterpret_cast<uint32_t*>(packed + grp * (GS / 2));
#pragma unroll 2
    for (int b = 0; b < GS / 8; ++b) {
        uint32_t word = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float v = group_elem<GS>(w, numel, grp, b * 8 + k);
            const uint32_t q = static_cast<uint32_t>(clampf(rintf(__fadd_rn(__fdiv_rn(v, sf), zf)), 0.0f, kQmax));
            word |= q << (4 * k);
        }
        out[b] = word;
    }
}

// preq bias of one group as the reference's callers build it: -zero * scale in float32
// (symmetric: -7.5 * scale)
__device__ __forceinline__ float preq_bias(const uint16_t* scales, const uint16_t* zeros, long long i, float* s_out) {
    const float s = __half2float(__ushort_as_half(scales[i]));
    *s_out = s;
    const float z = zeros ? __half2float(__ushort_as_half(zeros[i])) : 7.5f;
    return __fmul_rn(-z, s);
}

// QuantizedTensor (gs 32) -> preq2 meta [M][ng][4] + quant [ceil(M/4)][ng][4][16]: one thread per
// (band row, group); rows past M in the last band are zero (repack_preq2.py:31-44).
__global__ void k_pack_preq2(const uint8_t* __restrict__ packed, const uint16_t* __restrict__ scales,
                             const uint16_t* __restrict__ zeros, int M, int K, uint8_t* __restrict__ meta,
                             uint8_t* __restrict__ quant) {
    const int ng = K / 32;
    const long long nb = (M + 3) / 4;
    const long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= nb * 4 * ng) return;
    const long long row = t / ng;
    const int g = static_cast<int>(t - row * ng);
    uint4 nib = make_uint4(0u, 0u, 0u, 0u);
    if (row < M) {
        const long long i = row * ng + g;
        float s;
        const float bias = preq_bias(scales, zeros, i, &s);
        // repack_q4_32.py:84-97: scale = max(float(s), 1e-8), zero = -bias / scale in float64
        const double s64 = fmax(static_cast<double>(s), 1e-8);
        const double z64 = __ddiv_rn(-static_cast<double>(bias), s64);
        const uint32_t m = static_cast<uint32_t>(f16_bits_from_double(s64)) |
                           (static_cast<uint32_t>(f16_bits_from_double(z64)) << 16);
        reinterpret_cast<uint32_t*>(meta)[i] = m;
        nib = *reinterpret_cast<const uint4*>(packed + i * 16);
    }
    const long long band = row >> 2;
    *reinterpret_cast<uint4*>(quant + (band * ng + g) * 64 + (row & 3) * 16) = nib;
}

// Q4_128 block of 128 float32 weights (repack_q4_128.py:22-31): scale = fp16(amax / 7) and
// codes round(w * fl32(7 / amax)) + 8 clamped to [0, 15], amax and the divisions in float64;
// an all-(near-)zero group (amax < 1e-12) is scale 0, nibbles 0x88.
template <typename Src>
__device__ __forceinline__ void q4_128_block(Src src, uint8_t* __restrict__ blk) {
    float amax = 0.0f;
#pragma unroll 8
    for (int i = 0; i < 128; ++i) amax = fmaxf(amax, fabsf(src(i)));
    const double a64 = static_cast<double>(amax);
    uint16_t* out = reinterpret_cast<uint16_t*>(blk);  // 66-byte blocks start on even bytes
    if (a64 < 1e-12) {
        out[0] = 0;
        for (int b = 0; b < 32; ++b) out[1 + b] = 0x8888;
        return;
    }
    out[0] = f16_bits_from_double(__ddiv_rn(a64, 7.0));
    const float inv = __double2float_rn(__ddiv_rn(7.0, a64));
    for (int b = 0; b < 32; ++b) {
        uint32_t v = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float q = clampf(__fadd_rn(rintf(__fmul_rn(src(b * 4 + k), inv)), 8.0f), 0.0f, 15.0f);
            v |= static_cast<uint32_t>(q) << (4 * k);
        }
        out[1 + b] = static_cast<uint16_t>(v);
    }
}

// fp32 [M][K] -> Q4_128 blocks [M][K/128][66] (repack_fp32_to_q4_128_blocks): one warp per
// 128-float group, lane l owning elements 4l..4l+3 (one coalesced 512-byte read per group; the
// maximum by shuffles is the same value as the sequential one, fmaxf being exact), then the
// per-element arithmetic of q4_128_block, lane l writing nibble word l
__global__ void k_q4_128_from_f32(const float* __restrict__ w, int M, int K, uint8_t* __restrict__ blocks) {
    const int ng = K / 128;
    const long long n = static_cast<long long>(M) * ng;
    const int lane = threadIdx.x & 31;
    const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
    const bool vec = (reinterpret_cast<uintptr_t>(w) & 15u) == 0;
    for (long long t = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); t < n;
         t += warps) {
        const float* src = w + t * 128 + lane * 4;  // row r group g starts at r*K + g*128 = t*128
        float v[4];
        if (vec) {
            const float4 f = __ldg(reinterpret_cast<const float4*>(src));
            v[0] = f.x;
            v[1] = f.y;
            v[2] = f.z;
            v[3] = f.w;
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = __ldg(src + k);
        }
        float amax = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) amax = fmaxf(amax, fabsf(v[k]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const double a64 = static_cast<double>(amax);
        uint16_t* out = reinterpret_cast<uint16_t*>(blocks + t * 66);  // 66-byte blocks start on even bytes
        if (a64 < 1e-12) {
            if (lane == 0) out[0] = 0;
            out[1 + lane] = 0x8888;
            continue;
        }
        if (lane == 0) out[0] = f16_bits_from_double(__ddiv_rn(a64, 7.0));
        const float inv = __double2float_rn(__ddiv_rn(7.0, a64));
        uint32_t word = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float q = clampf(__fadd_rn(rintf(__fmul_rn(v[k], inv)), 8.0f), 0.0f, 15.0f);
            word |= static_cast<uint32_t>(q) << (4 * k);
        }
        out[1 + lane] = static_cast<uint16_t>(word);
    }
}

// gs-32 QuantizedTensor -> float32 q * scale + bias (phi4_cpu_run.py:3432-3448) -> Q4_128 blocks:
// the C0.1 requant of gate_up / down (build_c01_gs128_blocks)
__global__ void k_q4_128_from_quant(const uint8_t* __restrict__ packed, const uint16_t* __restrict__ scales,
                                    const uint16_t* __restrict__ zeros, int M, int K, uint8_t* __restrict__ blocks) {
    const int ng = K / 128;
    const long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= static_cast<long long>(M) * ng) return;
    const long long row = t / ng;
    const int g = static_cast<int>(t - row * ng);
    const long long g32 = row * (K / 32) + g * 4;  // first of the four gs-32 groups
    float sc[4], bi[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) bi[j] = preq_bias(scales, zeros, g32 + j, &sc[j]);
    const uint8_t* p = packed + (row * K + g * 128) / 2;
    q4_128_block(
        [&](int i) {
            const uint32_t byte = __ldg(p + (i >> 1));
            const float q = static_cast<float>((i & 1) ? (byte >> 4) : (byte & 15u));
            return __fadd_rn(__fmul_rn(q, sc[i >> 5]), bi[i >> 5]);
        },
        blocks + t * 66);
}

}  // namespace asdsl
