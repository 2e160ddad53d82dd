// gemv_stream.cuh -- the W4A8 / W4A32 decode GEMV family on sm_100a.
//
// One kernel template serves every weight format of the reference's decode
// path.  A weight matrix is a set of byte "streams" (preq2: quant + meta;
// packed: nibbles + scales + biases; the block formats: one stream), each made
// of fixed-size "units" (a 4-row band for preq2, one row otherwise).  Each CTA
// owns a contiguous run of units, so each of its streams is ONE contiguous
// span of HBM; a single producer thread walks that span with 1-D bulk copies
// (cp.async.bulk, no multicast) into a ring of shared-memory stages guarded by
// mbarriers, and consumer warps decode nibbles in registers, dot them against
// the int8 activation with dp4a, and apply the per-group fp32 combine.
//
// The activation prologue (A8 quantization, optionally preceded by RMSNorm) is
// fused: every CTA quantizes the whole input vector into shared memory while
// its first weight copies are in flight.  Epilogues: plain store, in-place
// residual add, paired gate/up SiLU*up, and per-CTA argmax with a last-CTA
// reduction.
//
// Reference formats and math (asdsl/kernels/native/):
//   preq2  gemv_preq2_avx2.cpp:196-297    preq   gemv_q4_preq_restored.cpp:305-473
//   Q4_128 gemv_q4_128.cpp:94-257          S256   gemv_q4_s256.cpp:83-209
//   Q4_K   gemv_q4_avx2.cpp:283-420        packed gemv_q4_avx2.cpp:665-749
#pragma once

#include "common.cuh"

namespace asdsl {

enum WeightFormat : int {
    kFmtPreq2 = 0,   // meta [M][ng][4] + quant [ceil(M/4)][ng][64], gs 32
    kFmtPreq = 1,    // [M][ng][20] blocks, gs 32
    kFmtQ4_128 = 2,  // [M][K/128][66] blocks, symmetric, implicit zero 8
    kFmtS256 = 3,    // [M][K/256][144] blocks, 8 fp16 sub-scales, zero 8, A8 gs 32
    kFmtQ4K = 4,     // [M][K/256][144] reference-interpretation Q4_K, own A8
    kFmtPacked = 5,  // nibbles [M][K/2] + fp32 scales [M][ng] + fp32 biases [M][ng], fp32 x
};

enum Prologue : int {
    kProA8 = 0,     // fp32 x -> A8 (gs 32 or 128)
    kProQ8 = 1,     // caller-quantized x (int8 + per-group fp32 scale)
    kProRmsA8 = 2,  // RMSNorm(x) * w then A8
    kProQ4K = 3,    // the Q4_K kernel's own A8 (half-away, clamp +-127)
    kProF32 = 4,    // fp32 x kept as is, plus per-group sums (packed W4A32)
};

enum Epilogue : int {
    kEpiStore = 0,   // y[row] = v
    kEpiResid = 1,   // resid[row] += v (in place; the decode residual stream)
    kEpiSilu = 2,    // paired gate/up: h[i] = silu(gate_i) * up_i
    kEpiArgmax = 3,  // y[row] = v (optional) + global first-max argmax
};

constexpr int kConsumerWarps = 8;
constexpr int kThreads = 32 * (kConsumerWarps + 1);  // + one producer warp
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kMaxStages = 16;
constexpr int kMaxStreams = 3;

struct StreamDesc {
    const uint8_t* base;   // 16-byte aligned
    long long unit_bytes;  // bytes per unit
    long long total_bytes; // stream length (clamps the last unit)
    uint32_t region_off;   // offset of this stream's region inside a segment of a stage
    uint32_t pad;
};

struct PipeArgs {
    StreamDesc s[kMaxStreams];
    int n_streams;
    int n_units;          // units per segment
    int pair_unit_off;    // > 0: paired (gate/up) mode, segment 1 starts this many units later
    int units_per_chunk;
    int n_stages;
    uint32_t seg_bytes;   // bytes of one segment inside a stage
    uint32_t stage_bytes; // bytes of one stage (1 or 2 segments)
    uint32_t xarea_off;   // dynamic smem offsets
    uint32_t stage_off;
};

struct GemvArgs {
    const float* x;        // fp32 activation
    const int8_t* xq;      // kProQ8: int8 activation
    const float* xs_in;    // kProQ8: per-group scales
    const float* norm_w;   // kProRmsA8
    float eps;
    int K;                 // in_features
    int M;                 // out rows (per segment)
    int gs;                // activation group size (32, or 128 for Q4_128)
    float* y;
    float* resid;
    float* h;
    // argmax (kEpiArgmax)
    float* part_val;
    int* part_idx;
    unsigned int* counter;
    float* out_val;
    int* out_idx;
    int row_base;          // global index of row 0 (row-sharded lm_head)
    unsigned int* status;  // device status word
};

// ---------------------------------------------------------------------------
// chunk geometry (shared by producer and consumers)
// ---------------------------------------------------------------------------
struct Span {
    long long a0;      // aligned start of the bulk copy (multiple of 16)
    long long a1;      // aligned end of the bulk copy (a1 >= a0)
    long long start;   // first byte of the chunk's data
    long long end;     // one past the last byte of the chunk's data
};

__device__ __forceinline__ Span chunk_span(const StreamDesc& sd, long long u_begin, long long u_end) {
    Span sp;
    sp.start = u_begin * sd.unit_bytes;
    sp.end = u_end * sd.unit_bytes;
    if (sp.end > sd.total_bytes) sp.end = sd.total_bytes;
    if (sp.start > sp.end) sp.start = sp.end;
    sp.a0 = sp.start & ~15ll;
    const long long tot16 = sd.total_bytes & ~15ll;
    long long a1 = (sp.end + 15) & ~15ll;
    if (a1 > tot16) a1 = tot16;
    if (a1 < sp.a0) a1 = sp.a0;
    sp.a1 = a1;
    return sp;
}

// ---------------------------------------------------------------------------
// activation prologue: x -> shared memory
// x8 (permuted per 32-group), xs[ng], xsi[ng] (int sums), xss[ng] (sum*scale)
// or, for kProF32, xf[K] floats + sx[ng] group sums.
// Runs on the consumer warps only; `nthreads` = consumer threads.
// ---------------------------------------------------------------------------
struct XArea {
    int8_t* x8;
    float* xs;
    int* xsi;
    float* xss;
    float* xf;
    float* sx;
    float* red;  // reduction scratch (kConsumerWarps floats)
};

__device__ __forceinline__ XArea xarea_layout(uint8_t* base, int K, int pro, int gs) {
    XArea a;
    const int ng = K / gs;
    if (pro == kProF32) {
        a.xf = reinterpret_cast<float*>(base);
        a.sx = a.xf + K;
        a.red = a.sx + ng;
        a.x8 = nullptr;
        a.xs = nullptr;
        a.xsi = nullptr;
        a.xss = nullptr;
    } else {
        a.x8 = reinterpret_cast<int8_t*>(base);
        a.xs = reinterpret_cast<float*>(base + ((K + 15) & ~15));
        a.xsi = reinterpret_cast<int*>(a.xs + ng);
        a.xss = reinterpret_cast<float*>(a.xsi + ng);
        a.red = a.xss + ng;
        a.xf = nullptr;
        a.sx = nullptr;
    }
    return a;
}

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

// Fused activation prologue.  The A8 rounding is the reference's compiled
// rounding (see common.cuh); with gs = 128 each 128-group is quantized as one
// group but stored as four permuted 32-records.
template <int PRO>
__device__ void run_prologue(const GemvArgs& ga, XArea xa, int cw, int lane) {
    const int K = ga.K;
    const int gs = ga.gs;
    const int ng = K / gs;
    const int ctid = cw * 32 + lane;
    const int nthr = kConsumerWarps * 32;

    if constexpr (PRO == kProF32) {
        for (int i = ctid; i < K; i += nthr) xa.xf[i] = __ldg(ga.x + i);
        consumer_sync();
        // group sums in the reference's 8-lane order (gemv_q4_avx2.cpp:677-685)
        for (int g = ctid; g < ng; g += nthr) {
            float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int j = 0; j < gs; j += 8)
#pragma unroll
                for (int l = 0; l < 8; ++l) lanes[l] = __fadd_rn(lanes[l], xa.xf[g * gs + j + l]);
            float a4[4];
#pragma unroll
            for (int l = 0; l < 4; ++l) a4[l] = __fadd_rn(lanes[l], lanes[l + 4]);
            xa.sx[g] = __fadd_rn(__fadd_rn(a4[0], a4[1]), __fadd_rn(a4[2], a4[3]));
        }
        consumer_sync();
        return;
    } else {
        float inv_rms = 1.0f;
        if constexpr (PRO == kProRmsA8) {
            // sum of squares -> inv = 1/sqrt(sum/n + eps)  (unified_engine.cpp:499-513)
            float ss = 0.0f;
            for (int i = ctid; i < K; i += nthr) {
                const float v = __ldg(ga.x + i);
                ss = __fmaf_rn(v, v, ss);
            }
            ss = warp_sum(ss);
            if (lane == 0) xa.red[cw] = ss;
            consumer_sync();
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) tot = __fadd_rn(tot, xa.red[w]);
            inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(K)), ga.eps)));
        }
        // one warp per 32-element sub-group; groups of 128 reduce over 4 warps' worth
        // of sub-groups, so iterate by activation group and let each lane own
        // gs/32 elements.
        const int sub = gs / 32;  // 1 or 4
        for (int g = cw; g < ng; g += kConsumerWarps) {
            float v[4];
            float amax = 0.0f;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                if (s < sub) {
                    const int idx = g * gs + s * 32 + lane;
                    float t;
                    if constexpr (PRO == kProQ8) {
                        t = 0.0f;
                    } else {
                        t = __ldg(ga.x + idx);
                        if constexpr (PRO == kProRmsA8) t = __fmul_rn(__fmul_rn(t, inv_rms), __ldg(ga.norm_w + idx));
                    }
                    v[s] = t;
                    amax = fmaxf(amax, fabsf(t));
                } else {
                    v[s] = 0.0f;
                }
            }
            int qs[4];
            float scale;
            if constexpr (PRO == kProQ8) {
                scale = __ldg(ga.xs_in + g);
#pragma unroll
                for (int s = 0; s < 4; ++s) qs[s] = (s < sub) ? static_cast<int>(__ldg(ga.xq + g * gs + s * 32 + lane)) : 0;
            } else if constexpr (PRO == kProQ4K) {
                // gemv_q4_avx2.cpp:377-400: amax < 1e-12 -> scale 0, codes 0;
                // q = clamp(round_half_away(x * 127/amax), -127, 127)
                amax = warp_max(amax);
                if (amax < 1e-12f) {
                    scale = 0.0f;
#pragma unroll
                    for (int s = 0; s < 4; ++s) qs[s] = 0;
                } else {
                    const float inv = __fdiv_rn(127.0f, amax);
                    scale = __fmul_rn(amax, inv127f());
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        int q = static_cast<int>(roundf(__fmul_rn(v[s], inv)));
                        q = q > 127 ? 127 : (q < -127 ? -127 : q);
                        qs[s] = q;
                    }
                }
            } else {
                amax = warp_max(amax);
                if (amax < 1e-9f) {
                    scale = 1.0f;
#pragma unroll
                    for (int s = 0; s < 4; ++s) qs[s] = 0;
                } else {
                    const float inv = __fdiv_rn(127.0f, amax);
                    scale = __fmul_rn(amax, inv127f());
#pragma unroll
                    for (int s = 0; s < 4; ++s) qs[s] = a8_code(v[s], inv);
                }
            }
            int qsum = 0;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                if (s < sub) {
                    xa.x8[(g * sub + s) * 32 + x8_perm_offset(lane)] = static_cast<int8_t>(qs[s]);
                    qsum += qs[s];
                }
            }
            qsum = warp_sum_i(qsum);
            if (lane == 0) {
                xa.xs[g] = scale;
                xa.xsi[g] = qsum;
                xa.xss[g] = __fmul_rn(static_cast<float>(qsum), scale);
            }
        }
        consumer_sync();
    }
}

// ---------------------------------------------------------------------------
// per-unit compute.  Each returns the row values for the unit in lanes:
//   preq2: lanes 0..3 hold rows band*4 + lane (after reduction)
//   row formats: all lanes hold the row value (after reduction)
// ---------------------------------------------------------------------------

// preq2 band: lane -> (group g0 + lane/4, row slot lane%4)
__device__ __forceinline__ float unit_preq2(const uint8_t* q, const uint8_t* m, int ng, const XArea& xa,
                                            int lane) {
    const int slot = lane & 3;
    const int gl = lane >> 2;
    float acc = 0.0f, corr = 0.0f;
    const uint8_t* mrow = m + slot * ng * 4;
    for (int g0 = 0; g0 < ng; g0 += 8) {
        const int g = g0 + gl;
        if (g < ng) {
            const uint4 w = *reinterpret_cast<const uint4*>(q + g * 64 + slot * 16);
            const uint32_t mw = *reinterpret_cast<const uint32_t*>(mrow + g * 4);
            const uint4 xa4 = *reinterpret_cast<const uint4*>(xa.x8 + g * 32);
            const uint4 xb4 = *reinterpret_cast<const uint4*>(xa.x8 + g * 32 + 16);
            const int d = dot_nib32(w, xa4, xb4, 0);
            const float ws = half_bits_to_float(mw);
            const float wz = half_bits_to_float(mw >> 16);
            const float comb = __fmul_rn(ws, xa.xs[g]);
            acc = __fmaf_rn(static_cast<float>(d), comb, acc);
            corr = __fmaf_rn(__fmul_rn(wz, ws), xa.xss[g], corr);
        }
    }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        acc += __shfl_xor_sync(0xffffffffu, acc, o);
        corr += __shfl_xor_sync(0xffffffffu, corr, o);
    }
    return acc - corr;
}

// preq row: 20-byte blocks at 4-byte aligned addresses; lane -> group
__device__ __forceinline__ float unit_preq(const uint8_t* row, int ng, const XArea& xa, int lane) {
    float acc = 0.0f, corr = 0.0f;
    for (int g = lane; g < ng; g += 32) {
        const uint32_t* b = reinterpret_cast<const uint32_t*>(row + g * 20);
        const uint32_t m = b[0];
        const uint4 w = make_uint4(b[1], b[2], b[3], b[4]);
        const uint4 xa4 = *reinterpret_cast<const uint4*>(xa.x8 + g * 32);
        const uint4 xb4 = *reinterpret_cast<const uint4*>(xa.x8 + g * 32 + 16);
        const int d = dot_nib32(w, xa4, xb4, 0);
        const float ws = half_bits_to_float(m), wz = half_bits_to_float(m >> 16);
        const float xs = xa.xs[g];
        acc = __fmaf_rn(static_cast<float>(d), __fmul_rn(ws, xs), acc);
        corr = __fadd_rn(corr, __fmul_rn(__fmul_rn(__fmul_rn(wz, static_cast<float>(xa.xsi[g])), ws), xs));
    }
    acc = warp_sum(acc);
    corr = warp_sum(corr);
    return acc - corr;
}

// Q4_128 row: 66-byte blocks; 4 lanes per block (16 nibble bytes each)
__device__ __forceinline__ float unit_q4_128(const uint8_t* row, int ng, const XArea& xa, int lane) {
    const int c = lane & 3;
    float acc = 0.0f, corr = 0.0f;
    for (int g0 = 0; g0 < ng; g0 += 8) {
        const int g = g0 + (lane >> 2);
        int d = 0;
        float comb = 0.0f;
        if (g < ng) {
            const uint8_t* blk = row + g * 66;
            const uint4 w = lds128_a2(blk + 2 + c * 16);
            const int8_t* xr = xa.x8 + (g * 4 + c) * 32;
            d = dot_nib32(w, *reinterpret_cast<const uint4*>(xr), *reinterpret_cast<const uint4*>(xr + 16), 0);
            const uint16_t sb = *reinterpret_cast<const uint16_t*>(blk);
            comb = __fmul_rn(half_bits_to_float(sb), xa.xs[g]);
        }
        d += __shfl_xor_sync(0xffffffffu, d, 1);
        d += __shfl_xor_sync(0xffffffffu, d, 2);
        if (g < ng && c == 0) {
            acc = __fmaf_rn(static_cast<float>(d), comb, acc);
            corr = __fmaf_rn(__fmul_rn(8.0f, static_cast<float>(xa.xsi[g])), comb, corr);
        }
    }
    acc = warp_sum(acc);
    corr = warp_sum(corr);
    return acc - corr;
}

// S256 row: 144-byte super-blocks, lane -> 32-weight sub-block
__device__ __forceinline__ float unit_s256(const uint8_t* row, int nsb, const XArea& xa, int lane) {
    float acc = 0.0f, corr = 0.0f;
    const int nsub = nsb * 8;
    for (int t = lane; t < nsub; t += 32) {
        const int sb = t >> 3, k = t & 7;
        const uint8_t* blk = row + sb * 144;
        const uint4 w = *reinterpret_cast<const uint4*>(blk + 16 + k * 16);
        const uint16_t sh = *reinterpret_cast<const uint16_t*>(blk + 2 * k);
        const int8_t* xr = xa.x8 + t * 32;
        const int d = dot_nib32(w, *reinterpret_cast<const uint4*>(xr), *reinterpret_cast<const uint4*>(xr + 16), 0);
        const float sc = __fmul_rn(half_bits_to_float(sh), xa.xs[t]);
        acc = __fmaf_rn(static_cast<float>(d), sc, acc);
        corr = __fmaf_rn(__fmul_rn(8.0f, static_cast<float>(xa.xsi[t])), sc, corr);
    }
    acc = warp_sum(acc);
    corr = warp_sum(corr);
    return acc - corr;
}

// Q4_K row (reference interpretation, gemv_q4_avx2.cpp:283-329)
__device__ __forceinline__ int get6_bits(const uint8_t* p, int idx) {
    const int bit = idx * 6, byte = bit >> 3, off = bit & 7;
    const int lo = p[byte];
    if (off <= 2) return (lo >> off) & 0x3F;
    return ((lo >> off) | (p[byte + 1] << (8 - off))) & 0x3F;
}

__device__ __forceinline__ float unit_q4k(const uint8_t* row, int nb, const XArea& xa, int lane) {
    float acc = 0.0f;
    const int nsub = nb * 8;
    for (int t = lane; t < nsub; t += 32) {
        const int b = t >> 3, sb = t & 7;
        const uint8_t* blk = row + b * 144;
        const uint32_t dd = *reinterpret_cast<const uint32_t*>(blk);
        const float d = half_bits_to_float(dd), dmin = half_bits_to_float(dd >> 16);
        const float sub_scale = __fmul_rn(d, static_cast<float>(get6_bits(blk + 4, sb)));
        const float sub_min = __fmul_rn(dmin, static_cast<float>(get6_bits(blk + 4, sb + 8)));
        const uint4 w = *reinterpret_cast<const uint4*>(blk + 16 + sb * 16);
        const int8_t* xr = xa.x8 + t * 32;
        const int dot = dot_nib32(w, *reinterpret_cast<const uint4*>(xr), *reinterpret_cast<const uint4*>(xr + 16), 0);
        const float part = __fsub_rn(__fmul_rn(sub_scale, static_cast<float>(dot)),
                                     __fmul_rn(sub_min, static_cast<float>(xa.xsi[t])));
        acc = __fmaf_rn(part, xa.xs[t], acc);
    }
    return warp_sum(acc);
}

// packed W4A32 row (no activation quantization): y = sum_g dot_f32 * s + b * sum(x_g)
__device__ __forceinline__ float unit_packed(const uint8_t* wrow, const float* srow, const float* brow, int K,
                                             int gs, const XArea& xa, int lane) {
    // lane -> 8 consecutive weights (4 bytes) per step; groups are gs/8 lanes wide
    const int ng = K / gs;
    float acc = 0.0f;
    const int lanes_per_group = gs / 8;  // gs multiple of 8 (checked on host)
    for (int base = 0; base < K; base += 256) {
        const int k = base + lane * 8;
        float d = 0.0f;
        int g = -1;
        if (k < K) {
            const uint32_t w = *reinterpret_cast<const uint32_t*>(wrow + (k >> 1));
            const float* xp = xa.xf + k;
#pragma unroll
            for (int e = 0; e < 8; ++e) d = __fmaf_rn(static_cast<float>((w >> (4 * e)) & 0xF), xp[e], d);
            g = k / gs;
        }
        // combine lanes of the same group (groups never straddle a 256-weight step
        // when 256 % gs == 0; otherwise fall back to per-lane scaling)
        if ((256 % gs) == 0 && lanes_per_group <= 32) {
            for (int o = 1; o < lanes_per_group; o <<= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
            if (g >= 0 && (lane % lanes_per_group) == 0)
                acc += __fmaf_rn(d, srow[g], __fmul_rn(brow[g], xa.sx[g]));
        } else if (g >= 0) {
            acc = __fmaf_rn(d, srow[g], acc);
            if ((k % gs) == 0) acc = __fmaf_rn(brow[g], xa.sx[g], acc);
        }
    }
    (void)ng;
    return warp_sum(acc);
}

// the reference's fast_exp_avx2 (unified_engine.cpp:803-825), scalar restatement
__device__ __forceinline__ float ref_fast_exp(float x) {
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
    return __fmul_rn(p, __int_as_float((i + 127) << 23));
}

// SiLU(g)*u as swiglu_inplace (unified_engine.cpp:836-856)
__device__ __forceinline__ float ref_silu_mul(float g, float u) {
    const float e = ref_fast_exp(__fsub_rn(0.0f, g));
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
    return __fmul_rn(__fmul_rn(g, sig), u);
}

// first-max argmax combine: larger value wins, ties go to the lower index
__device__ __forceinline__ void argmax_take(float& bv, int& bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int FMT, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, 1) k_stream_gemv(const PipeArgs pa, const GemvArgs ga) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    uint8_t* stages = smem + pa.stage_off;
    const int S = pa.n_stages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const long long U = pa.n_units;
    const long long u0 = U * blockIdx.x / gridDim.x;
    const long long u1 = U * (blockIdx.x + 1) / gridDim.x;
    const int CU = pa.units_per_chunk;
    const int n_chunks = static_cast<int>((u1 - u0 + CU - 1) / CU);
    const int nseg = pa.pair_unit_off > 0 ? 2 : 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kProducerWarp) {
        if (lane != 0) return;
        const uint64_t pol = l2_policy_evict_first();
        int issued = 0;
        bool ok = true;
        for (int j = 0; j < n_chunks; ++j) {
            const int s = j % S;
            const int use = j / S;
            if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) {
                atomicOr(ga.status, kStatusWaitEmpty);
                ok = false;
                break;
            }
            const long long cb = u0 + static_cast<long long>(j) * CU;
            const long long ce = (cb + CU < u1) ? cb + CU : u1;
            uint32_t tx = 0;
            for (int seg = 0; seg < nseg; ++seg)
                for (int i = 0; i < pa.n_streams; ++i) {
                    const Span sp = chunk_span(pa.s[i], cb + seg * pa.pair_unit_off, ce + seg * pa.pair_unit_off);
                    tx += static_cast<uint32_t>(sp.a1 - sp.a0);
                }
            mbar_arrive_expect_tx(&full[s], tx);
            uint8_t* st = stages + static_cast<size_t>(s) * pa.stage_bytes;
            for (int seg = 0; seg < nseg; ++seg)
                for (int i = 0; i < pa.n_streams; ++i) {
                    const Span sp = chunk_span(pa.s[i], cb + seg * pa.pair_unit_off, ce + seg * pa.pair_unit_off);
                    if (sp.a1 > sp.a0)
                        bulk_g2s_stream(st + seg * pa.seg_bytes + pa.s[i].region_off, pa.s[i].base + sp.a0,
                                        static_cast<uint32_t>(sp.a1 - sp.a0), &full[s], pol);
                }
            issued = j + 1;
        }
        // drain: never leave the CTA with copies in flight
        const int first = issued > S ? issued - S : 0;
        for (int j = first; j < issued; ++j) {
            if (!mbar_wait(&full[j % S], (j / S) & 1)) {
                atomicOr(ga.status, kStatusWaitDrain);
                break;
            }
        }
        (void)ok;
        return;
    }

    // ---------------- consumer warps ----------------
    const int cw = warp;
    XArea xa = xarea_layout(smem + pa.xarea_off, ga.K, PRO, ga.gs);
    run_prologue<PRO>(ga, xa, cw, lane);

    const int K = ga.K;
    const int M = ga.M;
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;

    for (int j = cw; j < n_chunks; j += kConsumerWarps) {
        const int s = j % S;
        const int use = j / S;
        if (!mbar_wait(&full[s], use & 1)) {
            if (lane == 0) atomicOr(ga.status, kStatusWaitFull);
            break;
        }
        const long long cb = u0 + static_cast<long long>(j) * CU;
        const long long ce = (cb + CU < u1) ? cb + CU : u1;
        uint8_t* st = stages + static_cast<size_t>(s) * pa.stage_bytes;

        // bytes past the last 16-byte boundary of a stream arrive by plain loads
        bool wrote_tail = false;
        for (int seg = 0; seg < nseg; ++seg)
            for (int i = 0; i < pa.n_streams; ++i) {
                const Span sp = chunk_span(pa.s[i], cb + seg * pa.pair_unit_off, ce + seg * pa.pair_unit_off);
                const long long t0 = sp.a1 > sp.start ? sp.a1 : sp.start;
                if (sp.end > t0) {
                    uint8_t* dst = st + seg * pa.seg_bytes + pa.s[i].region_off + (t0 - sp.a0);
                    const int nt = static_cast<int>(sp.end - t0);
                    if (lane < nt) dst[lane] = pa.s[i].base[t0 + lane];
                    wrote_tail = true;
                }
            }
        if (wrote_tail) {
            fence_proxy_async_smem();
            __syncwarp();
        }

        // data pointers for unit k of segment seg, stream i
        auto uptr = [&](int seg, int i, long long k) -> const uint8_t* {
            const Span sp = chunk_span(pa.s[i], cb + seg * pa.pair_unit_off, ce + seg * pa.pair_unit_off);
            return st + seg * pa.seg_bytes + pa.s[i].region_off + (sp.start - sp.a0) + k * pa.s[i].unit_bytes;
        };

        for (long long k = 0; k < ce - cb; ++k) {
            const long long unit = cb + k;
            float v[2];
            for (int seg = 0; seg < nseg; ++seg) {
                if constexpr (FMT == kFmtPreq2) {
                    v[seg] = unit_preq2(uptr(seg, 0, k), uptr(seg, 1, k), K / 32, xa, lane);
                } else if constexpr (FMT == kFmtPreq) {
                    v[seg] = unit_preq(uptr(seg, 0, k), K / 32, xa, lane);
                } else if constexpr (FMT == kFmtQ4_128) {
                    v[seg] = unit_q4_128(uptr(seg, 0, k), K / 128, xa, lane);
                } else if constexpr (FMT == kFmtS256) {
                    v[seg] = unit_s256(uptr(seg, 0, k), K / 256, xa, lane);
                } else if constexpr (FMT == kFmtQ4K) {
                    v[seg] = unit_q4k(uptr(seg, 0, k), K / 256, xa, lane);
                } else {
                    v[seg] = unit_packed(uptr(seg, 0, k), reinterpret_cast<const float*>(uptr(seg, 1, k)),
                                         reinterpret_cast<const float*>(uptr(seg, 2, k)), K, ga.gs, xa, lane);
                }
            }
            // rows of this unit and the lanes that own them
            long long row;
            bool own;
            if constexpr (FMT == kFmtPreq2) {
                row = unit * 4 + lane;
                own = lane < 4 && row < M;
            } else {
                row = unit;
                own = lane == 0 && row < M;
            }
            if (own) {
                if constexpr (EPI == kEpiStore) {
                    ga.y[row] = v[0];
                } else if constexpr (EPI == kEpiResid) {
                    ga.resid[row] = __fadd_rn(v[0], ga.resid[row]);
                } else if constexpr (EPI == kEpiSilu) {
                    ga.h[row] = ref_silu_mul(v[0], v[1]);
                } else {
                    if (ga.y) ga.y[row] = v[0];
                    argmax_take(best_v, best_i, v[0], ga.row_base + static_cast<int>(row));
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }

    if constexpr (EPI == kEpiArgmax) {
        // warp -> CTA -> grid (last CTA reduces the per-CTA partials)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
            argmax_take(best_v, best_i, ov, oi);
        }
        __shared__ float s_v[kConsumerWarps];
        __shared__ int s_i[kConsumerWarps];
        __shared__ bool s_last;
        if (lane == 0) {
            s_v[cw] = best_v;
            s_i[cw] = best_i;
        }
        consumer_sync();
        if (cw == 0 && lane == 0) {
            float bv = s_v[0];
            int bi = s_i[0];
            for (int w = 1; w < kConsumerWarps; ++w) argmax_take(bv, bi, s_v[w], s_i[w]);
            ga.part_val[blockIdx.x] = bv;
            ga.part_idx[blockIdx.x] = bi;
            __threadfence();
            const unsigned int prev = atomicAdd(ga.counter, 1u);
            s_last = (prev == gridDim.x - 1);
        }
        consumer_sync();
        if (s_last && cw == 0) {
            __threadfence();
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int b = lane; b < static_cast<int>(gridDim.x); b += 32)
                argmax_take(bv, bi, __ldcg(ga.part_val + b), __ldcg(ga.part_idx + b));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                argmax_take(bv, bi, ov, oi);
            }
            if (lane == 0) {
                *ga.out_val = bv;
                *ga.out_idx = (bi == 0x7fffffff) ? ga.row_base : bi;
                *ga.counter = 0u;  // re-arm for the next call
            }
        }
    }
}

}  // namespace asdsl
