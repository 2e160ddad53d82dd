/*
 * asdsl_oracle.c -- CPU restatement (plain C) of the reference's W4A8 decode
 * hot path.  TEST INFRASTRUCTURE ONLY: the checker for the CUDA kernels, never
 * part of the product.  Built by oracle/Makefile into oracle/liboracle.so.
 *
 * Compiled without fast-math and with -ffp-contract=off, so every rounding
 * below is the one written; FMAs are explicit (fmaf) where the reference uses
 * an FMA intrinsic.  Two places follow what the reference's *compiled* code
 * does under its own -ffast-math build (setup.py:56-65), which we pinned by
 * running the reference compiled here (oracle/_ref):
 *   - `amax / 127.0f` and `amax / 7.0f` are emitted by GCC as a multiply by
 *     the rounded reciprocal constant (reciprocal math), so the A8 scale is
 *     amax * fl(1/127) and the engine lm_head scale is amax * fl(1/7);
 *   - `127.0f / amax` and `7.0f / amax` stay true IEEE divisions.
 * The decode engine's path (the preq2 GEMV, RMSNorm, SwiGLU, attention) is
 * restated in the exact operation order of the reference's compiled code, so
 * this oracle's engine is bit-identical to the reference's UnifiedEngine
 * (tests/test_oracle_exact.py checks that against oracle/_ref):
 *   - the preq2 GEMV keeps the 8 int32 lanes of each group's dot product
 *     (pmaddubsw + pmaddwd lanes: elements 4j..4j+3) as 8 float accumulators
 *     per even/odd group, and ends with (hsum(even) + hsum(odd)) - (corr_even
 *     + corr_odd), the order GCC emits for gemv_preq2_avx2.cpp:250;
 *   - `1.0f / std::sqrt(a)` (RMSNorm, attention's 1/sqrt(head_dim)) is emitted
 *     as RSQRTSS plus one Newton step, (x0*(a*x0) - 3) * (x0 * -0.5), and the
 *     vector divide of SwiGLU's sigmoid as RCPPS plus one Newton step,
 *     (x0 + x0) - x0*(x0*d); both estimates come from this host's CPU, like the
 *     reference's;
 *   - RMSNorm's per-element product is (x*w)*inv, SwiGLU's (g*u)*sigmoid, and
 *     1 + p*2^i is one FMA; attention's num*old_scale + tile_num is one FMA.
 * The other GEMV formats keep the reference's structure (even/odd group
 * accumulators, 8-lane partial sums) where that is cheap to restate; their
 * remaining fp32 reassociation differences are covered by the 1e-3 tolerance.
 */
#include "asdsl_oracle.h"

#include <xmmintrin.h>

#include <math.h>
#include <stdlib.h>
#include <string.h>

static const float kInv127 = 1.0f / 127.0f; /* constant-folded, as GCC does */
static const float kInv7 = 1.0f / 7.0f;

static inline float h2f(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}
static inline uint16_t f2h(float f) {
    _Float16 v = (_Float16)f; /* IEEE round-to-nearest-even */
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}
static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* The host CPU's approximate reciprocal instructions, as the reference's compiled code runs them,
 * and GCC's one-step Newton refinements of them under -ffast-math (operand order as emitted). */
static inline float x86_rsqrt(float a) { return _mm_cvtss_f32(_mm_rsqrt_ss(_mm_set_ss(a))); }
static inline float x86_rcp(float a) { return _mm_cvtss_f32(_mm_rcp_ss(_mm_set_ss(a))); }
float or_host_rcp(float a) { return x86_rcp(a); }
float or_host_rsqrt(float a) { return x86_rsqrt(a); }
/* the C library's expf over an array (the reference's attention calls it, unified_engine.cpp:989) */
void or_expf_array(const float* x, float* y, long n) {
#pragma omp parallel for schedule(static)
    for (long i = 0; i < n; ++i) y[i] = expf(x[i]);
}
float or_nr_rsqrt(float a) {
    const float x0 = x86_rsqrt(a);
    const float t = fmaf(x0, x0 * a, -3.0f);
    return t * (x0 * -0.5f);
}
float or_nr_recip(float d) {
    const float x0 = x86_rcp(d);
    const float e = x0 * (x0 * d);
    return (x0 + x0) - e;
}
/* hsum256_ps (unified_engine.cpp:152-161): ((v0+v4)+(v1+v5)) + ((v2+v6)+(v3+v7)) */
static inline float hsum8(const float v[8]) {
    return ((v[0] + v[4]) + (v[1] + v[5])) + ((v[2] + v[6]) + (v[3] + v[7]));
}

/* ---------------------------------------------------------------------------
 * A8: asdsl/kernels/native/gemv_q4_preq_restored.cpp:505-549
 *   per group: amax; amax < 1e-9 -> q = 0, scale = 1.0;
 *   else scale = amax * fl(1/127), inv = 127/amax, q = RNE(x*inv) saturated.
 * xsum (int32 sum of q per group) as compute_x_sums_scaled, gemv_preq2_avx2.cpp:70-93.
 * ------------------------------------------------------------------------- */
void or_quantize_activation(const float* x, int8_t* xq, float* xs, int32_t* xsum, int K, int gs) {
    const int ng = K / gs;
    for (int g = 0; g < ng; ++g) {
        const float* xg = x + (long)g * gs;
        int8_t* q = xq + (long)g * gs;
        float amax = 0.0f;
        for (int j = 0; j < gs; ++j) {
            float a = fabsf(xg[j]);
            if (a > amax) amax = a;
        }
        int32_t s = 0;
        if (amax < 1e-9f) {
            memset(q, 0, (size_t)gs);
            xs[g] = 1.0f;
        } else {
            xs[g] = amax * kInv127;
            const float inv = 127.0f / amax;
            for (int j = 0; j < gs; ++j) {
                float r = rintf(xg[j] * inv);
                int v = (int)r;
                if (v > 127) v = 127;
                if (v < -128) v = -128;
                q[j] = (int8_t)v;
                s += v;
            }
        }
        if (xsum) xsum[g] = s;
    }
}

/* Q4_K A8: gemv_q4_avx2.cpp:374-402 (half-away rounding, clamp +-127,
 * amax < 1e-12 -> scale 0). */
void or_quantize_activation_q4k(const float* x, int8_t* xq, float* xs, int K) {
    const int ng = K / 32;
    for (int g = 0; g < ng; ++g) {
        const float* xg = x + g * 32;
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) {
            float a = fabsf(xg[i]);
            if (a > amax) amax = a;
        }
        if (amax < 1e-12f) {
            xs[g] = 0.0f;
            memset(xq + g * 32, 0, 32);
            continue;
        }
        const float inv = 127.0f / amax;
        xs[g] = amax * kInv127;
        for (int i = 0; i < 32; ++i) {
            int v = (int)roundf(xg[i] * inv);
            if (v > 127) v = 127;
            if (v < -127) v = -127;
            xq[g * 32 + i] = (int8_t)v;
        }
    }
}

/* int dot of 32 nibbles (16 bytes, low nibble = even index) with 32 int8 */
static inline int32_t dot32(const uint8_t* nib, const int8_t* xq) {
    int32_t d = 0;
    for (int b = 0; b < 16; ++b) {
        d += (int32_t)(nib[b] & 0x0F) * xq[2 * b];
        d += (int32_t)(nib[b] >> 4) * xq[2 * b + 1];
    }
    return d;
}
static inline int32_t sum32(const int8_t* q) {
    int32_t s = 0;
    for (int i = 0; i < 32; ++i) s += q[i];
    return s;
}

/* preq2: gemv_preq2_avx2.cpp:196-253 (process_one_row, the OpenMP row loop at :289-292), in the
 * compiled operation order.  Per group g: combined = ws*xs; corr_term = (wz*ws)*xsum_scaled;
 * lane j of the int32 dot (pmaddubsw + pmaddwd: elements 4j..4j+3) -> term_j = (float)dot_j *
 * combined, added to lane j of the even or odd accumulator; corr_term to the even or odd scalar.
 * y = (hsum(acc_even) + hsum(acc_odd)) - (corr_even + corr_odd). */
void or_gemv_preq2_q8(const uint8_t* meta, const uint8_t* quant, const int8_t* xq, const float* xs,
                      float* y, int M, int K) {
    const int ng = K / 32;
    float* xsum_scaled = (float*)malloc(sizeof(float) * (size_t)ng);
    for (int g = 0; g < ng; ++g) xsum_scaled[g] = (float)sum32(xq + g * 32) * xs[g];
#pragma omp parallel for schedule(static)
    for (int r = 0; r < M; ++r) {
        const uint8_t* mrow = meta + (size_t)r * ng * 4;
        const uint8_t* qband = quant + (size_t)(r / 4) * ng * 64 + (r % 4) * 16;
        float acc[2][8] = {{0}}, corr[2] = {0.0f, 0.0f};
        for (int g = 0; g < ng; ++g) {
            const float ws = h2f(rd16(mrow + g * 4));
            const float wz = h2f(rd16(mrow + g * 4 + 2));
            const float comb = ws * xs[g];
            const float ct = (wz * ws) * xsum_scaled[g];
            const uint8_t* nib = qband + (size_t)g * 64;
            const int8_t* xg = xq + g * 32;
            for (int j = 0; j < 8; ++j) {
                const int32_t d = (int32_t)(nib[2 * j] & 0x0F) * xg[4 * j] + (int32_t)(nib[2 * j] >> 4) * xg[4 * j + 1] +
                                  (int32_t)(nib[2 * j + 1] & 0x0F) * xg[4 * j + 2] +
                                  (int32_t)(nib[2 * j + 1] >> 4) * xg[4 * j + 3];
                acc[g & 1][j] += (float)d * comb;
            }
            corr[g & 1] += ct;
        }
        y[r] = (hsum8(acc[0]) + hsum8(acc[1])) - (corr[0] + corr[1]);
    }
    free(xsum_scaled);
}

void or_gemv_preq2_fused(const uint8_t* meta, const uint8_t* quant, const float* x, float* y, int M, int K) {
    int8_t* xq = (int8_t*)malloc((size_t)K);
    float* xs = (float*)malloc(sizeof(float) * (size_t)(K / 32));
    or_quantize_activation(x, xq, xs, NULL, K, 32);
    or_gemv_preq2_q8(meta, quant, xq, xs, y, M, K);
    free(xq);
    free(xs);
}

/* preq 20-byte blocks: gemv_q4_preq_restored.cpp:318-336 per group
 * (acc += dot*(ws*xs); corr += wz*xsum*ws*xs), y = acc - corr (:417-419). */
void or_gemv_preq_q8(const uint8_t* blocks, const int8_t* xq, const float* xs, float* y, int M, int K) {
    const int ng = K / 32;
    int32_t* xsum = (int32_t*)malloc(sizeof(int32_t) * (size_t)ng);
    for (int g = 0; g < ng; ++g) xsum[g] = sum32(xq + g * 32);
#pragma omp parallel for schedule(static)
    for (int r = 0; r < M; ++r) {
        const uint8_t* row = blocks + (size_t)r * ng * 20;
        float acc = 0.0f, corr = 0.0f;
        for (int g = 0; g < ng; ++g) {
            const uint8_t* b = row + g * 20;
            const float ws = h2f(rd16(b)), wz = h2f(rd16(b + 2));
            acc += (float)dot32(b + 4, xq + g * 32) * (ws * xs[g]);
            corr += wz * (float)xsum[g] * ws * xs[g];
        }
        y[r] = acc - corr;
    }
    free(xsum);
}

/* Q4_128 66-byte blocks: gemv_q4_128.cpp:122-147 (one_row):
 * combined = ws*xs; acc += dot*combined; corr += 8*xsum*combined. */
void or_gemv_q4_128_q8(const uint8_t* blocks, const int8_t* xq, const float* xs, float* y, int M, int K) {
    const int ng = K / 128;
    int32_t* xsum = (int32_t*)malloc(sizeof(int32_t) * (size_t)ng);
    for (int g = 0; g < ng; ++g) {
        int32_t s = 0;
        for (int i = 0; i < 128; ++i) s += xq[g * 128 + i];
        xsum[g] = s;
    }
#pragma omp parallel for schedule(static)
    for (int r = 0; r < M; ++r) {
        const uint8_t* row = blocks + (size_t)r * ng * 66;
        float acc = 0.0f, corr = 0.0f;
        for (int g = 0; g < ng; ++g) {
            const uint8_t* b = row + g * 66;
            const float comb = h2f(rd16(b)) * xs[g];
            int32_t d = 0;
            for (int c = 0; c < 4; ++c) d += dot32(b + 2 + c * 16, xq + g * 128 + c * 32);
            acc += (float)d * comb;
            corr += 8.0f * (float)xsum[g] * comb;
        }
        y[r] = acc - corr;
    }
    free(xsum);
}

/* Batched prompt GEMM on fp32 activations (gemm_q4_128_q8_avx2, gemv_q4_128.cpp:262-306): per
 * (row, 128-group) the weights dequantized exactly, w = ((q & 15) - 8) * ws; per batch row an
 * 8-lane fma dot over the group (lane j takes elements j, j+8, ...), folded as
 * (l0+l4 + l1+l5) + (l2+l6 + l3+l7) (hsum256_q4128, :49-58), added to that row's accumulator.
 * Only batch rows b < 64 are computed; y rows b >= 64 are left as they are.  gs != 128 -> -1. */
int or_gemm_q4_128_f32(const uint8_t* blocks, const float* x, float* y, int M, int K, int gs, int batch) {
    if (gs != 128) return -1;
    const int ng = K / 128;
    const int nb = batch < 64 ? batch : 64;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < M; ++r) {
        const uint8_t* row = blocks + (size_t)r * ng * 66;
        float acc[64];
        for (int b = 0; b < nb; ++b) acc[b] = 0.0f;
        for (int g = 0; g < ng; ++g) {
            const uint8_t* blk = row + g * 66;
            const float ws = h2f(rd16(blk));
            float wf[128];
            for (int i = 0; i < 64; ++i) {
                const uint8_t v = blk[2 + i];
                wf[2 * i] = (float)((v & 0x0F) - 8) * ws;
                wf[2 * i + 1] = (float)((v >> 4) - 8) * ws;
            }
            for (int b = 0; b < nb; ++b) {
                const float* xb = x + (size_t)b * K + g * 128;
                float l[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                for (int i = 0; i < 128; i += 8)
                    for (int j = 0; j < 8; ++j) l[j] = fmaf(wf[i + j], xb[i + j], l[j]);
                const float h0 = l[0] + l[4], h1 = l[1] + l[5], h2 = l[2] + l[6], h3 = l[3] + l[7];
                acc[b] += (h0 + h1) + (h2 + h3);
            }
        }
        for (int b = 0; b < nb; ++b) y[(size_t)b * M + r] = acc[b];
    }
    return 0;
}

/* Q4_S256: gemv_q4_s256.cpp:110-138: 8 fp16 sub-scales + 128 nibble bytes,
 * activations at gs 32; acc += dot*(ws*xs), corr += 8*xsum*(ws*xs). */
void or_gemv_q4_s256_q8(const uint8_t* blocks, const int8_t* xq, const float* xs, float* y, int M, int K) {
    const int nsb = K / 256, ng = K / 32;
    int32_t* xsum = (int32_t*)malloc(sizeof(int32_t) * (size_t)ng);
    for (int g = 0; g < ng; ++g) xsum[g] = sum32(xq + g * 32);
#pragma omp parallel for schedule(static)
    for (int r = 0; r < M; ++r) {
        const uint8_t* row = blocks + (size_t)r * nsb * 144;
        float acc = 0.0f, corr = 0.0f;
        for (int sb = 0; sb < nsb; ++sb) {
            const uint8_t* b = row + sb * 144;
            for (int k = 0; k < 8; ++k) {
                const int g = sb * 8 + k;
                const float sc = h2f(rd16(b + 2 * k)) * xs[g];
                acc += (float)dot32(b + 16 + k * 16, xq + g * 32) * sc;
                corr += 8.0f * (float)xsum[g] * sc;
            }
        }
        y[r] = acc - corr;
    }
    free(xsum);
}

/* 6-bit little-endian bitstream read: gemv_q4_avx2.cpp:110-120 */
static inline int get6(const uint8_t* p, int idx) {
    const int bit = idx * 6, byte = bit >> 3, off = bit & 7;
    if (off <= 2) return (p[byte] >> off) & 0x3F;
    return ((p[byte] >> off) | (p[byte + 1] << (8 - off))) & 0x3F;
}

/* Q4_K (reference interpretation): gemv_q4_avx2.cpp:283-329 per super-block;
 * acc += (d*sc*dot - dmin*m*xsum) * xs per 32-sub-block. */
void or_gemv_q4km(const uint8_t* w, const float* x, float* y, int M, int K) {
    const int nb = K / 256, ng = K / 32;
    int8_t* xq = (int8_t*)malloc((size_t)K);
    float* xs = (float*)malloc(sizeof(float) * (size_t)ng);
    or_quantize_activation_q4k(x, xq, xs, K);
#pragma omp parallel for schedule(static)
    for (int r = 0; r < M; ++r) {
        const uint8_t* row = w + (size_t)r * nb * 144;
        float acc = 0.0f;
        for (int b = 0; b < nb; ++b) {
            const uint8_t* blk = row + b * 144;
            const float d = h2f(rd16(blk)), dmin = h2f(rd16(blk + 2));
            float bacc = 0.0f;
            for (int sb = 0; sb < 8; ++sb) {
                const float sub_scale = d * (float)get6(blk + 4, sb);
                const float sub_min = dmin * (float)get6(blk + 4, sb + 8);
                const int8_t* q = xq + b * 256 + sb * 32;
                const int32_t dot = dot32(blk + 16 + sb * 16, q);
                const int32_t xsum = sum32(q);
                bacc += (sub_scale * (float)dot - sub_min * (float)xsum) * xs[b * 8 + sb];
            }
            acc += bacc;
        }
        y[r] = acc;
    }
    free(xq);
    free(xs);
}

/* fp32-activation packed W4 GEMV (no A8): gemv_q4_avx2.cpp:665-749;
 * y = sum_g dot_f32(q, x_g) * scale + bias * sum(x_g). */
void or_gemv_q4_packed(const uint8_t* w, const float* x, const float* scales, const float* biases,
                       float* y, int M, int K, int gs) {
    const int ng = K / gs;
    float* sx = (float*)malloc(sizeof(float) * (size_t)ng);
    for (int g = 0; g < ng; ++g) {
        float s = 0.0f;
        for (int j = 0; j < gs; ++j) s += x[g * gs + j];
        sx[g] = s;
    }
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m) {
        const uint8_t* row = w + (size_t)m * (K / 2);
        float acc = 0.0f;
        for (int g = 0; g < ng; ++g) {
            float d = 0.0f;
            for (int j = 0; j < gs; ++j) {
                const int k = g * gs + j;
                const int q = (k & 1) ? (row[k >> 1] >> 4) : (row[k >> 1] & 0x0F);
                d = fmaf((float)q, x[k], d);
            }
            const size_t gi = (size_t)m * ng + g;
            acc += d * scales[gi] + biases[gi] * sx[g];
        }
        y[m] = acc;
    }
    free(sx);
}

/* Engine lm_head symmetric Q4_32 -> preq2: unified_engine.cpp:320-400.
 * amax < 1e-12 -> scale bits 0, zero 0x4800, nibbles 0x88;
 * else scale = fp16_rne(amax * fl(1/7)), zero = fp16(8.0) = 0x4800,
 * q = clamp(round_half_away(x * (7/amax)) + 8, 0, 15). */
void or_lmhead_quant_q4_32_preq2(const uint16_t* wf16, uint8_t* meta, uint8_t* quant, int rows, int cols) {
    const int ng = cols / 32;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        float xg[32];
        for (int g = 0; g < ng; ++g) {
            float amax = 0.0f;
            for (int j = 0; j < 32; ++j) {
                xg[j] = h2f(wf16[(size_t)r * cols + g * 32 + j]);
                float a = fabsf(xg[j]);
                if (a > amax) amax = a;
            }
            uint8_t* m = meta + ((size_t)r * ng + g) * 4;
            uint8_t* q = quant + ((size_t)(r / 4) * ng + g) * 64 + (r % 4) * 16;
            if (amax < 1e-12f) {
                m[0] = 0; m[1] = 0; m[2] = 0x00; m[3] = 0x48;
                memset(q, 0x88, 16);
                continue;
            }
            const uint16_t sf = f2h(amax * kInv7);
            m[0] = (uint8_t)(sf & 0xFF); m[1] = (uint8_t)(sf >> 8);
            m[2] = 0x00; m[3] = 0x48;
            const float inv = 7.0f / amax;
            for (int j = 0; j < 32; j += 2) {
                int q0 = (int)roundf(xg[j] * inv) + 8, q1 = (int)roundf(xg[j + 1] * inv) + 8;
                q0 = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
                q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
                q[j / 2] = (uint8_t)((q1 << 4) | q0);
            }
        }
    }
}

/* Engine lm_head Q4_128: unified_engine.cpp:411-461 (same rules, 66-byte blocks). */
void or_lmhead_quant_q4_128(const uint16_t* wf16, uint8_t* blocks, int rows, int cols) {
    const int ng = cols / 128;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        float xg[128];
        for (int g = 0; g < ng; ++g) {
            float amax = 0.0f;
            for (int j = 0; j < 128; ++j) {
                xg[j] = h2f(wf16[(size_t)r * cols + g * 128 + j]);
                float a = fabsf(xg[j]);
                if (a > amax) amax = a;
            }
            uint8_t* b = blocks + ((size_t)r * ng + g) * 66;
            if (amax < 1e-12f) {
                b[0] = 0; b[1] = 0;
                memset(b + 2, 0x88, 64);
                continue;
            }
            const uint16_t sf = f2h(amax * kInv7);
            b[0] = (uint8_t)(sf & 0xFF); b[1] = (uint8_t)(sf >> 8);
            const float inv = 7.0f / amax;
            for (int j = 0; j < 128; j += 2) {
                int q0 = (int)roundf(xg[j] * inv) + 8, q1 = (int)roundf(xg[j + 1] * inv) + 8;
                q0 = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
                q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
                b[2 + j / 2] = (uint8_t)((q1 << 4) | q0);
            }
        }
    }
}

/* ---------------------------------------------------------------------------
 * Engine ops, unified_engine.cpp
 * ------------------------------------------------------------------------- */

/* :499-524  inv = 1/sqrt(sum/n + eps); out = (x*inv)*w  (8-lane FMA partials) */
static float sumsq8(const float* x, int n) {
    float lane[8] = {0};
    int i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) lane[l] = fmaf(x[i + l], x[i + l], lane[l]);
    /* hsum256_ps order: (lo+hi) then pairwise */
    float a[4];
    for (int l = 0; l < 4; ++l) a[l] = lane[l] + lane[l + 4];
    float s = (a[0] + a[1]) + (a[2] + a[3]);
    for (; i < n; ++i) s += x[i] * x[i];
    return s;
}

/* compiled order: inv = nr_rsqrt(sum/n + eps) (RSQRTSS + Newton), out = (x*w)*inv */
void or_rmsnorm(float* out, const float* in, const float* w, int n, float eps) {
    const float s = sumsq8(in, n);
    const float inv = or_nr_rsqrt(s / (float)n + eps);
    for (int i = 0; i < n; ++i) out[i] = (in[i] * w[i]) * inv;
}

/* :663-693 */
void or_residual_add_rmsnorm(float* hidden, float* residual, const float* w, int n, float eps) {
    for (int i = 0; i < n; ++i) {
        const float v = hidden[i] + residual[i];
        hidden[i] = v;
        residual[i] = v;
    }
    or_rmsnorm(hidden, hidden, w, n, eps);
}

/* :768-801 pairs (i, i+half); o0 = fma(xf, c, -(xs*s)), o1 = fma(xf, s, xs*c) */
void or_rope(float* q, float* k, const float* cos_t, const float* sin_t, int pos, int rotary_dim,
             int n_heads, int n_kv_heads, int head_dim) {
    const int half = rotary_dim / 2;
    const float* c = cos_t + (size_t)pos * half;
    const float* s = sin_t + (size_t)pos * half;
    for (int h = 0; h < n_heads + n_kv_heads; ++h) {
        float* row = (h < n_heads) ? q + (size_t)h * head_dim : k + (size_t)(h - n_heads) * head_dim;
        for (int i = 0; i < half; ++i) {
            const float xf = row[i], xs = row[half + i];
            row[i] = fmaf(xf, c[i], -(xs * s[i]));
            row[half + i] = fmaf(xf, s[i], xs * c[i]);
        }
    }
}

/* swiglu_inplace :836-857 (vector path: size is a multiple of 8) with fast_exp_avx2 (:803-825)
 * inlined, in the compiled order: d = fma(p, 2^i, 1) (the multiply by 2^i and the add contracted),
 * sigmoid = RCPPS(d) + one Newton step, val = (g*u)*sigmoid. */
void or_swiglu(float* gate, const float* up, int n) {
    for (int i = 0; i < n; ++i) {
        const float g = gate[i];
        float x = -g;
        x = fmaxf(x, -87.3f);
        x = fminf(x, 87.3f);
        x = x * 1.4426950408889634f;
        const float fi = rintf(x);
        const int k = (int)fi;
        const float f = x - fi;
        float p = fmaf(0.001333838100523091f, f, 0.009618129107628477f);
        p = fmaf(p, f, 0.05550410866482158f);
        p = fmaf(p, f, 0.2402265069591007f);
        p = fmaf(p, f, 0.6931471805599453f);
        p = fmaf(p, f, 1.0f);
        const uint32_t eb = (uint32_t)(k + 127) << 23;
        float e;
        memcpy(&e, &eb, 4);
        const float d = fmaf(p, e, 1.0f);
        gate[i] = (g * up[i]) * or_nr_recip(d);
    }
}

/* :207-233 first max wins */
int or_argmax(const float* v, int n) {
    if (n <= 0) return 0;
    int bi = 0;
    float bv = v[0];
    for (int i = 1; i < n; ++i)
        if (v[i] > bv) {
            bv = v[i];
            bi = i;
        }
    return bi;
}

/* :859-920 one position: per head per 64-block; scale = absmax*fl(1/127)
 * (or 1e-12), inv = 127/absmax (or 1e12), q = clamp(RNE(x*inv), -127, 127). */
void or_kv_write(int8_t* kq, float* ks, int8_t* vq, float* vs, const float* k, const float* v,
                 int n_kv_heads, int head_dim) {
    const int nbk = head_dim / 64;
    for (int h = 0; h < n_kv_heads; ++h)
        for (int b = 0; b < nbk; ++b) {
            const int off = h * head_dim + b * 64;
            float ka = 0.0f, va = 0.0f;
            for (int i = 0; i < 64; ++i) {
                ka = fmaxf(ka, fabsf(k[off + i]));
                va = fmaxf(va, fabsf(v[off + i]));
            }
            const float sk = ka > 1e-12f ? ka * kInv127 : 1e-12f;
            const float sv = va > 1e-12f ? va * kInv127 : 1e-12f;
            ks[h * nbk + b] = sk;
            vs[h * nbk + b] = sv;
            /* the compiled code folds 1/(absmax * fl(1/127)) into 127/absmax (reciprocal math);
             * the tiny-block branch multiplies by fl(1e12) */
            const float ik = ka > 1e-12f ? 127.0f / ka : 1e12f, iv = va > 1e-12f ? 127.0f / va : 1e12f;
            for (int i = 0; i < 64; ++i) {
                int a = (int)rintf(k[off + i] * ik), c = (int)rintf(v[off + i] * iv);
                a = a < -127 ? -127 : (a > 127 ? 127 : a);
                c = c < -127 ? -127 : (c > 127 ? 127 : c);
                kq[off + i] = (int8_t)a;
                vq[off + i] = (int8_t)c;
            }
        }
}

/* :922-1027 single-query GQA attention over int8 KV, online softmax in
 * 64-position tiles, scores * 1/sqrt(head_dim), libm exp.
 * kq/vq point at position 0 of this layer: element (pos, kvh, d) at
 * pos*pos_stride_q8 + kvh*head_dim + d; scales at pos*pos_stride_sc + kvh*(head_dim/64) + b. */
void or_attention(float* out, const float* q, const int8_t* kq, const float* ks, const int8_t* vq,
                  const float* vs, int seq_pos, int n_heads, int n_kv_heads, int head_dim,
                  long pos_stride_q8, long pos_stride_sc) {
    const int groups = n_heads / n_kv_heads > 0 ? n_heads / n_kv_heads : 1;
    const float inv_sqrt_d = or_nr_rsqrt((float)head_dim); /* RSQRTSS + Newton, as compiled */
    const int nbk = head_dim / 64;
    float* scores = (float*)malloc(sizeof(float) * 64);
    float* num = (float*)malloc(sizeof(float) * (size_t)head_dim);
    float* tnum = (float*)malloc(sizeof(float) * (size_t)head_dim);
    for (int h = 0; h < n_heads; ++h) {
        const int kvh = h / groups;
        const float* qh = q + (size_t)h * head_dim;
        memset(num, 0, sizeof(float) * (size_t)head_dim);
        float m = -INFINITY, l = 0.0f;
        for (int tk = 0; tk <= seq_pos; tk += 64) {
            const int kend = (seq_pos + 1 < tk + 64) ? seq_pos + 1 : tk + 64;
            const int span = kend - tk;
            float tmax = -INFINITY;
            for (int p = 0; p < span; ++p) {
                const long pos = tk + p;
                float dot = 0.0f;
                for (int b = 0; b < nbk; ++b) {
                    const float sc = ks[pos * pos_stride_sc + kvh * nbk + b];
                    const int8_t* kr = kq + pos * pos_stride_q8 + (long)kvh * head_dim + b * 64;
                    float lane[8] = {0};
                    for (int i = 0; i < 64; i += 8)
                        for (int t = 0; t < 8; ++t)
                            lane[t] = fmaf(qh[b * 64 + i + t], (float)kr[i + t] * sc, lane[t]);
                    float a4[4];
                    for (int t = 0; t < 4; ++t) a4[t] = lane[t] + lane[t + 4];
                    dot += (a4[0] + a4[1]) + (a4[2] + a4[3]);
                }
                scores[p] = dot * inv_sqrt_d;
                if (scores[p] > tmax) tmax = scores[p];
            }
            const float nm = m > tmax ? m : tmax;
            const float old_scale = (l > 0.0f) ? expf(m - nm) : 0.0f;
            float tl = 0.0f;
            memset(tnum, 0, sizeof(float) * (size_t)head_dim);
            for (int p = 0; p < span; ++p) {
                const long pos = tk + p;
                const float w = expf(scores[p] - nm);
                tl += w;
                for (int b = 0; b < nbk; ++b) {
                    const float sc = vs[pos * pos_stride_sc + kvh * nbk + b];
                    const int8_t* vr = vq + pos * pos_stride_q8 + (long)kvh * head_dim + b * 64;
                    for (int i = 0; i < 64; ++i) tnum[b * 64 + i] = fmaf(w, (float)vr[i] * sc, tnum[b * 64 + i]);
                }
            }
            m = nm;
            l = l * old_scale + tl;
            for (int i = 0; i < head_dim; ++i) num[i] = fmaf(num[i], old_scale, tnum[i]); /* contracted */
        }
        const float il = 1.0f / l;
        for (int i = 0; i < head_dim; ++i) out[(size_t)h * head_dim + i] = num[i] * il;
    }
    free(scores);
    free(num);
    free(tnum);
}

/* ---------------------------------------------------------------------------
 * Engine: UnifiedEngine::forward_token, unified_engine.cpp:1339-1688, C0 path
 * (fused_preq, preq2 blobs present, lm_head preq2 g32).
 * ------------------------------------------------------------------------- */
struct or_engine {
    or_model_t m;
    float *hidden, *residual, *qkv, *att, *gu;
    int8_t *kq, *vq;
    float *ks, *vs;
    long l_stride_q8, l_stride_sc;
};

or_engine_t* or_engine_create(const or_model_t* m) {
    or_engine_t* e = (or_engine_t*)calloc(1, sizeof(or_engine_t));
    e->m = *m;
    const int qd = m->n_heads * m->head_dim, kvd = m->n_kv_heads * m->head_dim;
    e->hidden = (float*)calloc((size_t)m->hidden, sizeof(float));
    e->residual = (float*)calloc((size_t)m->hidden, sizeof(float));
    e->qkv = (float*)calloc((size_t)(qd + 2 * kvd), sizeof(float));
    e->att = (float*)calloc((size_t)qd, sizeof(float));
    e->gu = (float*)calloc((size_t)m->inter * 2, sizeof(float));
    e->l_stride_q8 = (long)m->max_seq * kvd;
    e->l_stride_sc = (long)m->max_seq * m->n_kv_heads * (m->head_dim / 64);
    e->kq = (int8_t*)calloc((size_t)m->num_layers * e->l_stride_q8, 1);
    e->vq = (int8_t*)calloc((size_t)m->num_layers * e->l_stride_q8, 1);
    e->ks = (float*)calloc((size_t)m->num_layers * e->l_stride_sc, sizeof(float));
    e->vs = (float*)calloc((size_t)m->num_layers * e->l_stride_sc, sizeof(float));
    return e;
}

void or_engine_destroy(or_engine_t* e) {
    if (!e) return;
    free(e->hidden); free(e->residual); free(e->qkv); free(e->att); free(e->gu);
    free(e->kq); free(e->vq); free(e->ks); free(e->vs);
    free(e);
}

void or_engine_reset(or_engine_t* e) {
    memset(e->kq, 0, (size_t)e->m.num_layers * e->l_stride_q8);
    memset(e->vq, 0, (size_t)e->m.num_layers * e->l_stride_q8);
}

int or_engine_forward_token(or_engine_t* e, int token, int pos, float* logits) {
    const or_model_t* m = &e->m;
    if (token < 0 || token >= m->vocab || pos < 0 || pos >= m->max_seq) return 1;
    const int H = m->hidden, qd = m->n_heads * m->head_dim, kvd = m->n_kv_heads * m->head_dim;
    const int qkv_n = qd + 2 * kvd, nbk = m->head_dim / 64;
    for (int i = 0; i < H; ++i) e->hidden[i] = h2f(m->embed_f16[(size_t)token * H + i]); /* :181-197 */
    for (int l = 0; l < m->num_layers; ++l) {
        memcpy(e->residual, e->hidden, sizeof(float) * (size_t)H);                     /* :1378 */
        or_rmsnorm(e->hidden, e->hidden, m->rms_att[l], H, m->eps);                     /* :1380 */
        or_gemv_preq2_fused(m->qkv_meta[l], m->qkv_quant[l], e->hidden, e->qkv, qkv_n, H); /* :1411 */
        or_rope(e->qkv, e->qkv + qd, m->cos_t, m->sin_t, pos, m->rotary_dim,
                m->n_heads, m->n_kv_heads, m->head_dim);                                /* :1433 */
        int8_t* kq = e->kq + l * e->l_stride_q8;
        int8_t* vq = e->vq + l * e->l_stride_q8;
        float* ks = e->ks + l * e->l_stride_sc;
        float* vs = e->vs + l * e->l_stride_sc;
        or_kv_write(kq + (long)pos * kvd, ks + (long)pos * m->n_kv_heads * nbk,
                    vq + (long)pos * kvd, vs + (long)pos * m->n_kv_heads * nbk,
                    e->qkv + qd, e->qkv + qd + kvd, m->n_kv_heads, m->head_dim);       /* :1441 */
        or_attention(e->att, e->qkv, kq, ks, vq, vs, pos, m->n_heads, m->n_kv_heads, m->head_dim,
                     kvd, (long)m->n_kv_heads * nbk);                                   /* :1449 */
        or_gemv_preq2_fused(m->o_meta[l], m->o_quant[l], e->att, e->hidden, H, qd);     /* :1487 */
        or_residual_add_rmsnorm(e->hidden, e->residual, m->rms_ffn[l], H, m->eps);      /* :1508 */
        or_gemv_preq2_fused(m->gu_meta[l], m->gu_quant[l], e->hidden, e->gu, 2 * m->inter, H); /* :1539 */
        or_swiglu(e->gu, e->gu + m->inter, m->inter);                                   /* :1568 */
        or_gemv_preq2_fused(m->dn_meta[l], m->dn_quant[l], e->gu, e->hidden, H, m->inter); /* :1599 */
        for (int i = 0; i < H; ++i) e->hidden[i] += e->residual[i];                     /* :1623 */
    }
    if (logits) {
        or_rmsnorm(e->hidden, e->hidden, m->output_norm, H, m->eps);                    /* :1633 */
        or_gemv_preq2_fused(m->lm_meta, m->lm_quant, e->hidden, logits, m->vocab, H);   /* :1637 */
    }
    return 0;
}

/* 2-bit GEMVs of the QCSD draft bank (gemv_q2_avx2.cpp).  group_sum_x: eight interleaved lane
 * sums of x per group folded by hsum256_ps, plus the tail (:138-148, :62-73); per row and group the
 * dot of the codes with x, then row_sum += scale * dot + bias * group_sum_x (:154-173, :79-114).
 * packed: code j of a byte in bits 2j..2j+1, four codes per x chunk summed as written (:163-168);
 * unpacked: one code per byte, eight fma lanes folded by hsum256_ps plus the tail (:86-104). */
static void q2_group_sums(const float* x, int K, int gs, float* gsum) {
    const int ng = K / gs;
    for (int g = 0; g < ng; ++g) {
        const float* xg = x + g * gs;
        float l[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        int j = 0;
        for (; j + 8 <= gs; j += 8)
            for (int k = 0; k < 8; ++k) l[k] += xg[j + k];
        float sum = hsum8(l);
        for (; j < gs; ++j) sum += xg[j];
        gsum[g] = sum;
    }
}

void or_gemv_q2_packed(const uint8_t* w, const float* x, const float* scales, const float* biases, float* y,
                       int M, int K, int gs) {
    const int ng = K / gs, stride = K / 4;
    float* gsum = (float*)malloc(sizeof(float) * (size_t)ng);
    q2_group_sums(x, K, gs, gsum);
    for (int m = 0; m < M; ++m) {
        const uint8_t* row = w + (size_t)m * stride;
        float row_sum = 0.0f;
        for (int g = 0; g < ng; ++g) {
            const int k0 = g * gs;
            const size_t gi = (size_t)m * ng + g;
            float dot = 0.0f;
            for (int j = 0; j < gs; j += 4) {
                const uint8_t b = row[(k0 + j) / 4];
                const float v0 = (float)(b & 3), v1 = (float)((b >> 2) & 3), v2 = (float)((b >> 4) & 3),
                            v3 = (float)((b >> 6) & 3);
                dot += v0 * x[k0 + j] + v1 * x[k0 + j + 1] + v2 * x[k0 + j + 2] + v3 * x[k0 + j + 3];
            }
            row_sum += scales[gi] * dot + biases[gi] * gsum[g];
        }
        y[m] = row_sum;
    }
    free(gsum);
}

void or_gemv_q2_unpacked(const uint8_t* w, const float* x, const float* scales, const float* biases, float* y,
                         int M, int K, int gs) {
    const int ng = K / gs;
    float* gsum = (float*)malloc(sizeof(float) * (size_t)ng);
    q2_group_sums(x, K, gs, gsum);
    for (int m = 0; m < M; ++m) {
        const uint8_t* row = w + (size_t)m * K;
        float row_sum = 0.0f;
        for (int g = 0; g < ng; ++g) {
            const int k0 = g * gs;
            float l[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            int j = 0;
            for (; j + 8 <= gs; j += 8)
                for (int k = 0; k < 8; ++k) l[k] = fmaf((float)row[k0 + j + k], x[k0 + j + k], l[k]);
            float dot = hsum8(l);
            for (; j < gs; ++j) dot += (float)row[k0 + j] * x[k0 + j];
            row_sum += scales[(size_t)m * ng + g] * dot + biases[(size_t)m * ng + g] * gsum[g];
        }
        y[m] = row_sum;
    }
    free(gsum);
}
