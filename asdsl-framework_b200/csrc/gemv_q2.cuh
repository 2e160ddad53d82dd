// gemv_q2.cuh -- 2-bit fp32-activation GEMVs (the QCSD draft bank's kernels)
//
// Reference: gemv_q2_unpacked_impl / gemv_q2_packed_impl (asdsl/kernels/native/gemv_q2_avx2.cpp:
// 53-118, :128-174): y[m] = sum_g (scale[m,g] * dot_g + bias[m,g] * sum_x[g]) with dot_g the fp32
// dot of the group's 2-bit codes (0..3) with x and sum_x[g] the group's sum of x.  Unpacked
// weights hold one code per byte; packed ones four per byte, code j of a byte in bits 2j..2j+1.
//
// B200 form: x and the group sums are staged in shared memory once per CTA (the sums in the
// reference's order: eight interleaved lanes, then ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7))); a warp
// takes a row at a time and its lanes take consecutive groups, so a warp's weight reads are one
// contiguous run of the row; the lanes' partial sums meet in a shuffle reduction.  HBM bound:
// M*K/4 (packed) or M*K (unpacked) code bytes + 8 bytes of scale and bias per group.
// `accumulate` (the engine's draft step): y[m] += result, the residual add of o and down.
#pragma once

#include "common.cuh"

namespace asdsl {

constexpr int kQ2Warps = 8;

// 16 codes of one lane times x[k0 .. k0+15] from shared memory: four float4 loads, rotated by
// (lane / 2) so that the 8 lanes of a load phase hit 32 distinct banks
__device__ __forceinline__ float q2_dot16(const float* xs, int k0, const uint32_t (&c)[4], int lane, bool packed) {
    float d = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int q = (i + (lane >> 1)) & 3;  // float4 q of the lane's 16 x values
        const float4 xv = *reinterpret_cast<const float4*>(xs + k0 + 4 * q);
        uint32_t v[4];
        if (packed) {
            const uint32_t byte = (c[q >> 2] >> (8 * (q & 3))) & 0xFFu;  // c[0] holds all 16 codes
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = (byte >> (2 * k)) & 3u;
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = (c[q] >> (8 * k)) & 0xFFu;
        }
        d = __fmaf_rn(static_cast<float>(v[0]), xv.x, d);
        d = __fmaf_rn(static_cast<float>(v[1]), xv.y, d);
        d = __fmaf_rn(static_cast<float>(v[2]), xv.z, d);
        d = __fmaf_rn(static_cast<float>(v[3]), xv.w, d);
    }
    return d;
}

template <bool kPacked>
__global__ void __launch_bounds__(kQ2Warps * 32)
    k_gemv_q2(const uint8_t* __restrict__ w, const float* __restrict__ x, const float* __restrict__ scales,
              const float* __restrict__ biases, float* __restrict__ y, int M, int K, int gs, int accumulate) {
    extern __shared__ __align__(16) float q2_smem[];
    float* xs = q2_smem;        // [K]
    float* gsum = q2_smem + K;  // [K / gs]
    const int ng = K / gs;
    for (int i = threadIdx.x; i < K; i += blockDim.x) xs[i] = x[i];
    __syncthreads();
    for (int g = threadIdx.x; g < ng; g += blockDim.x) {
        const float* xg = xs + g * gs;
        float l[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        int j = 0;
        for (; j + 8 <= gs; j += 8)
#pragma unroll
            for (int k = 0; k < 8; ++k) l[k] = __fadd_rn(l[k], xg[j + k]);
        float sum = __fadd_rn(__fadd_rn(__fadd_rn(l[0], l[4]), __fadd_rn(l[1], l[5])),
                              __fadd_rn(__fadd_rn(l[2], l[6]), __fadd_rn(l[3], l[7])));
        for (; j < gs; ++j) sum = __fadd_rn(sum, xg[j]);
        gsum[g] = sum;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const long long row_bytes = kPacked ? K / 4 : K;
    // fast form: every lane takes 16 consecutive codes (one 32-bit word packed, one 16-byte word
    // unpacked), a group spans gs/16 adjacent lanes whose dots meet in shuffles
    const int lpg = gs / 16;
    const bool fast = (gs % 16) == 0 && lpg <= 32 && (32 % lpg) == 0 && (K % 16) == 0 &&
                      (reinterpret_cast<uintptr_t>(w) & 15u) == 0;
    for (int m = blockIdx.x * kQ2Warps + (threadIdx.x >> 5); m < M; m += gridDim.x * kQ2Warps) {
        const uint8_t* row = w + static_cast<long long>(m) * row_bytes;
        float acc = 0.0f;
        if (fast) {
            for (int k0 = lane * 16; k0 - lane * 16 < K; k0 += 512) {
                float dot = 0.0f;
                if (k0 < K) {
                    uint32_t c[4];
                    if constexpr (kPacked) {
                        c[0] = *reinterpret_cast<const uint32_t*>(row + k0 / 4);
                        c[1] = c[2] = c[3] = c[0];
                    } else {
                        const uint4 u = *reinterpret_cast<const uint4*>(row + k0);
                        c[0] = u.x;
                        c[1] = u.y;
                        c[2] = u.z;
                        c[3] = u.w;
                    }
                    dot = q2_dot16(xs, k0, c, lane, kPacked);
                }
                for (int o = 1; o < lpg; o <<= 1) dot = __fadd_rn(dot, __shfl_xor_sync(0xffffffffu, dot, o));
                if (k0 < K && (lane % lpg) == 0) {
                    const int g = k0 / gs;
                    const long long gi = static_cast<long long>(m) * ng + g;
                    acc = __fadd_rn(acc, __fmaf_rn(scales[gi], dot, __fmul_rn(biases[gi], gsum[g])));
                }
            }
        } else {
            for (int g = lane; g < ng; g += 32) {
                const float* xg = xs + g * gs;
                float dot = 0.0f;
                if constexpr (kPacked) {
                    const uint8_t* bg = row + g * (gs / 4);
                    for (int j = 0; j < gs / 4; ++j) {
                        const uint32_t b = bg[j];
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            dot = __fmaf_rn(static_cast<float>((b >> (2 * k)) & 3u), xg[4 * j + k], dot);
                    }
                } else {
                    const uint8_t* bg = row + g * gs;
                    for (int j = 0; j < gs; ++j) dot = __fmaf_rn(static_cast<float>(bg[j]), xg[j], dot);
                }
                const long long gi = static_cast<long long>(m) * ng + g;
                acc = __fadd_rn(acc, __fmaf_rn(scales[gi], dot, __fmul_rn(biases[gi], gsum[g])));
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) y[m] = accumulate ? __fadd_rn(y[m], acc) : acc;  // accumulate: the residual add
    }
}

}  // namespace asdsl
