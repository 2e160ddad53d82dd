// gemm_q4_128.cuh -- batched prompt GEMM over Q4_128 blocks with fp32 activations.
//
// Reference: gemm_q4_128_q8_avx2 (asdsl/kernels/native/gemv_q4_128.cpp:262-306), the GEMM the
// reference engine's forward_batch runs for its g128 projections (unified_engine.cpp:1154-1215).
// For every row and 128-group the weights are dequantized exactly, w = ((q & 15) - 8) * ws; per
// batch row b the group's dot is an 8-lane fma chain (lane j takes elements j, j+8, ..., j+120)
// folded as ((l0+l4) + (l1+l5)) + ((l2+l6) + (l3+l7)) (hsum256_q4128, :49-58) and added to the
// row's accumulator.  This kernel keeps that order, so its outputs are bit-identical.  Like the
// reference, only batch rows b < 64 are computed; Y rows b >= 64 are not written.
//
// Layout: one CTA of 8 warps per 32 rows; warp w owns rows 4w .. 4w+3 and lane l batch rows l and
// l + 32.  Per 128-group the CTA stages the batch's activations (transposed to [k/4][b] float4,
// padded to 65 columns so the staging writes and the compute reads are conflict-free) and its
// 32 rows' dequantized weights ([row][k/4] float4, read as broadcasts), then every thread runs
// its 4 x 2 eight-lane chains.  Weights are read from global memory once; the activations of the
// whole batch are re-read from L2 by every CTA.  (Fetching the next group during the compute --
// cp.async into a second activation tile, weight bytes into registers -- measured no faster on
// B200: it takes the kernel from 104 to 137 registers, one CTA per SM instead of two.)
#pragma once

#include "common.cuh"

namespace asdsl {

constexpr int kGemmRows = 32;        // rows per CTA
constexpr int kGemmMaxBatch = 64;    // batch rows the reference computes
constexpr int kGemmXPitch = kGemmMaxBatch + 1;  // float4 columns of the staged activation tile
constexpr size_t kGemmSmem = (32 * kGemmXPitch + kGemmRows * 32) * sizeof(float4);

__global__ void __launch_bounds__(256) k_gemm_q4_128_f32(const uint8_t* __restrict__ blocks,
                                                         const float* __restrict__ X, float* __restrict__ Y,
                                                         int M, int K, int B) {
    extern __shared__ float4 gsm[];
    float4* xs4 = gsm;                      // [32 k-quads][kGemmXPitch batch rows]
    float4* wf4 = gsm + 32 * kGemmXPitch;   // [kGemmRows rows][32 k-quads]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ng = K / 128;
    const int row0 = blockIdx.x * kGemmRows;
    const bool two = B > 32;  // uniform: a second batch row per lane
    float acc[4][2];
    float l[4][2][8];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int t = 0; t < 2; ++t) acc[r][t] = 0.0f;

    for (int g = 0; g < ng; ++g) {
        __syncthreads();  // the previous group's tiles are consumed
        // activations: warp w stages batch rows w, w + 8, ...; lane = k-quad (one 512-byte row read)
        for (int b = warp; b < B; b += 8)
            xs4[lane * kGemmXPitch + b] =
                __ldg(reinterpret_cast<const float4*>(X + static_cast<long long>(b) * K + g * 128) + lane);
        // weights: thread -> (row tid / 8, nibble bytes 8c .. 8c + 7 = elements 16c .. 16c + 15)
        {
            const int r = tid >> 3, c = tid & 7;
            const int row = row0 + r;
            float4 w[4] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f),
                           make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
            if (row < M) {
                const uint8_t* blk = blocks + (static_cast<long long>(row) * ng + g) * 66;
                const float ws = half_bits_to_float(*reinterpret_cast<const uint16_t*>(blk));
                const uint16_t* nb = reinterpret_cast<const uint16_t*>(blk + 2 + c * 8);
                float f[16];
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    const uint32_t v = nb[h];
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const uint32_t byte = (v >> (8 * j)) & 0xFFu;
                        f[4 * h + 2 * j] = __fmul_rn(static_cast<float>(static_cast<int>(byte & 0x0Fu) - 8), ws);
                        f[4 * h + 2 * j + 1] = __fmul_rn(static_cast<float>(static_cast<int>(byte >> 4) - 8), ws);
                    }
                }
#pragma unroll
                for (int h = 0; h < 4; ++h) w[h] = make_float4(f[4 * h], f[4 * h + 1], f[4 * h + 2], f[4 * h + 3]);
            }
#pragma unroll
            for (int h = 0; h < 4; ++h) wf4[r * 32 + c * 4 + h] = w[h];
        }
        __syncthreads();

#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int t = 0; t < 2; ++t)
#pragma unroll
                for (int j = 0; j < 8; ++j) l[r][t][j] = 0.0f;
        const float4* wrow = wf4 + (warp * 4) * 32;
        for (int kq2 = 0; kq2 < 16; ++kq2) {
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {  // k-quad 2 kq2 + hf: elements of lanes 4 hf .. 4 hf + 3
                const int kq = 2 * kq2 + hf;
                const float4 xa = xs4[kq * kGemmXPitch + lane];
                float4 xb = make_float4(0.f, 0.f, 0.f, 0.f);
                if (two) xb = xs4[kq * kGemmXPitch + lane + 32];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const float4 w = wrow[r * 32 + kq];
                    l[r][0][4 * hf + 0] = __fmaf_rn(w.x, xa.x, l[r][0][4 * hf + 0]);
                    l[r][0][4 * hf + 1] = __fmaf_rn(w.y, xa.y, l[r][0][4 * hf + 1]);
                    l[r][0][4 * hf + 2] = __fmaf_rn(w.z, xa.z, l[r][0][4 * hf + 2]);
                    l[r][0][4 * hf + 3] = __fmaf_rn(w.w, xa.w, l[r][0][4 * hf + 3]);
                    if (two) {
                        l[r][1][4 * hf + 0] = __fmaf_rn(w.x, xb.x, l[r][1][4 * hf + 0]);
                        l[r][1][4 * hf + 1] = __fmaf_rn(w.y, xb.y, l[r][1][4 * hf + 1]);
                        l[r][1][4 * hf + 2] = __fmaf_rn(w.z, xb.z, l[r][1][4 * hf + 2]);
                        l[r][1][4 * hf + 3] = __fmaf_rn(w.w, xb.w, l[r][1][4 * hf + 3]);
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const float h0 = __fadd_rn(l[r][t][0], l[r][t][4]), h1 = __fadd_rn(l[r][t][1], l[r][t][5]);
                const float h2 = __fadd_rn(l[r][t][2], l[r][t][6]), h3 = __fadd_rn(l[r][t][3], l[r][t][7]);
                acc[r][t] = __fadd_rn(acc[r][t], __fadd_rn(__fadd_rn(h0, h1), __fadd_rn(h2, h3)));
            }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int row = row0 + warp * 4 + r;
        if (row >= M) continue;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const int b = lane + 32 * t;
            if (b < B) Y[static_cast<long long>(b) * M + row] = acc[r][t];
        }
    }
}

}  // namespace asdsl
