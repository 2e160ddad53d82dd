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

template <bool kPacked>
__global__ void __launch_bounds__(kQ2Warps * 32)
    k_gemv_q2(const uint8_t* __restrict__ w, const float* __restrict__ x, const float* __restrict__ scales,
              const float* __restrict__ biases, float* __restrict__ y, int M, int K, int gs, int accumulate) {
    extern __shared__ float q2_smem[];
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
    for (int m = blockIdx.x * kQ2Warps + (threadIdx.x >> 5); m < M; m += gridDim.x * kQ2Warps) {
        const uint8_t* row = w + static_cast<long long>(m) * row_bytes;
        float acc = 0.0f;
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
        acc = warp_sum(acc);
        if (lane == 0) y[m] = accumulate ? __fadd_rn(y[m], acc) : acc;  // accumulate: the residual add
    }
}

}  // namespace asdsl
