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

constexpr int kQ2Warps = 16;

// 16 codes of one lane times x[k0 .. k0+15] from shared memory: four float4 loads, rotated by
// (lane / 2) so that the 8 lanes of a load phase hit 32 distinct banks
__device__ __forceinline__ float q2_dot16(const float* xs, int k0, const uint32_t (&c)[4], int lane, bool packed) {
    float d = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int q = (i + (lane >> 1)) & 3;  // float4 q of the lane's 16 x values
        const float4 xv = *reinterpret_cast<const float4*>(xs + k0 + 4 * q);
        // code -> float without the conversion pipe: the bits 0x4B000000 | c are the float 2^23 + c,
        // minus 2^23 exactly c
        float v[4];
        if (packed) {
            const uint32_t byte = (c[q >> 2] >> (8 * (q & 3))) & 0xFFu;  // c[0] holds all 16 codes
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = __fsub_rn(__uint_as_float(0x4B000000u | ((byte >> (2 * k)) & 3u)), 8388608.0f);
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = __fsub_rn(__uint_as_float(0x4B000000u | ((c[q] >> (8 * k)) & 0xFFu)), 8388608.0f);
        }
        d = __fmaf_rn(v[0], xv.x, d);
        d = __fmaf_rn(v[1], xv.y, d);
        d = __fmaf_rn(v[2], xv.z, d);
        d = __fmaf_rn(v[3], xv.w, d);
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
    const int lane = threadIdx.x & 31;
    // x -> shared memory (16-byte loads when aligned), then the group sums: eight lanes of a warp
    // per group, lane k summing x[8j + k] over j, folded by shuffles in hsum256_ps's order
    if ((K & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
        for (int i = threadIdx.x; i < K / 4; i += blockDim.x)
            reinterpret_cast<float4*>(xs)[i] = __ldg(reinterpret_cast<const float4*>(x) + i);
    } else {
        for (int i = threadIdx.x; i < K; i += blockDim.x) xs[i] = x[i];
    }
    __syncthreads();
    if ((gs & 7) == 0) {
        const int seg = lane >> 3, k = lane & 7;
        for (int g0 = (threadIdx.x >> 5) * 4; g0 < ng; g0 += kQ2Warps * 4) {
            const int g = g0 + seg;
            float l = 0.0f;
            if (g < ng)
                for (int j = 0; j < gs; j += 8) l = __fadd_rn(l, xs[g * gs + j + k]);
            const float a = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, 4));  // l_k + l_(k+4)
            const float b = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 1));  // (l0+l4)+(l1+l5), (l2+l6)+(l3+l7)
            const float c = __fadd_rn(b, __shfl_xor_sync(0xffffffffu, b, 2));
            if (g < ng && k == 0) gsum[g] = c;
        }
    } else {
        for (int g = threadIdx.x; g < ng; g += blockDim.x) {
            const float* xg = xs + g * gs;
            float l[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            int j = 0;
            for (; j + 8 <= gs; j += 8)
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) l[kk] = __fadd_rn(l[kk], xg[j + kk]);
            float sum = __fadd_rn(__fadd_rn(__fadd_rn(l[0], l[4]), __fadd_rn(l[1], l[5])),
                                  __fadd_rn(__fadd_rn(l[2], l[6]), __fadd_rn(l[3], l[7])));
            for (; j < gs; ++j) sum = __fadd_rn(sum, xg[j]);
            gsum[g] = sum;
        }
    }
    __syncthreads();
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
            // eight steps at a time (4096 codes): their code words, scales and biases are all
            // loaded first, so a warp keeps up to 4 KB of its row in flight
            constexpr int U = 8;
            for (int base = 0; base < K; base += U * 512) {
                uint32_t cw[U][4];
                float sc[U], bi[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int k0 = base + u * 512 + lane * 16;
                    sc[u] = bi[u] = 0.0f;
                    cw[u][0] = cw[u][1] = cw[u][2] = cw[u][3] = 0u;
                    if (k0 < K) {
                        if constexpr (kPacked) {
                            cw[u][0] = *reinterpret_cast<const uint32_t*>(row + k0 / 4);
                        } else {
                            const uint4 q = *reinterpret_cast<const uint4*>(row + k0);
                            cw[u][0] = q.x;
                            cw[u][1] = q.y;
                            cw[u][2] = q.z;
                            cw[u][3] = q.w;
                        }
                        const long long gi = static_cast<long long>(m) * ng + k0 / gs;
                        sc[u] = __ldg(scales + gi);
                        bi[u] = __ldg(biases + gi);
                    }
                }
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int k0 = base + u * 512 + lane * 16;
                    uint32_t c[4] = {cw[u][0], kPacked ? cw[u][0] : cw[u][1], kPacked ? cw[u][0] : cw[u][2],
                                     kPacked ? cw[u][0] : cw[u][3]};
                    float dot = (k0 < K) ? q2_dot16(xs, k0, c, lane, kPacked) : 0.0f;
                    for (int o = 1; o < lpg; o <<= 1) dot = __fadd_rn(dot, __shfl_xor_sync(0xffffffffu, dot, o));
                    if (k0 < K && (lane % lpg) == 0)
                        acc = __fadd_rn(acc, __fmaf_rn(sc[u], dot, __fmul_rn(bi[u], gsum[k0 / gs])));
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
