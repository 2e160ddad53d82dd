// attention_exact.cuh -- the decode attention of one layer in the reference's compiled order
// (reference-exact numerics mode).
//
// Reference: rope_apply_inplace (unified_engine.cpp:768-801), set_kv_cache (:859-920) and
// compute_attention_flash_q8 (:922-1027).  One CTA per query head, in the reference's order:
//   * RoPE pairs (i, i + rot/2): o0 = fma(x_first, c, -(x_second*s)), o1 = fma(x_first, s, x_second*c);
//   * int8 KV per 64-dim block: scale = absmax * fl(1/127) (1e-12 for a zero block), codes
//     RNE(x * 127/absmax) (the compiled code folds 1/scale into 127/absmax; 1e12 for a zero block)
//     clamped to +-127; the first head of a KV group stores them;
//   * score of position p: per 64-dim block, eight lanes l accumulate q[8i+l] * (k[8i+l]*scale) by
//     FMA over i, folded ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7)); dot = (0 + block0) + block1;
//     s = dot * inv_sqrt_d (RSQRTSS + Newton of head_dim, computed on the host);
//   * 64-position tiles in order: new_m = max(m, tile max); old = l > 0 ? expf(m - new_m) : 0;
//     w_p = expf(s_p - new_m) with the C library's expf; tile_l += w_p and
//     tile_num[d] = fma(w_p, v[d]*scale, tile_num[d]) in position order; l = l*old + tile_l
//     (two roundings); num[d] = fma(num[d], old, tile_num[d]);
//   * out[d] = num[d] * (1/l).
// Thread d < 128 owns dim d; every thread replays the (m, l) bookkeeping, so no broadcast is
// needed.  The scores of all positions live in shared memory (max_seq <= kAttnXMaxSeq).
#pragma once

#include "engine_ops.cuh"
#include "exact_math.cuh"

namespace asdsl {

constexpr int kAttnXThreads = 256;
constexpr int kAttnXMaxSeq = 4096;
constexpr int kAttnXTile = 64;

struct AttnXSmem {
    float q[kAttnHeadDim];
    float k[kAttnHeadDim];  // this position's dequantized k, v (what the cache read gives back)
    float v[kAttnHeadDim];
    float red[2][2][2];
    float w[kAttnXTile];
    float vs[kAttnXTile][2];
    alignas(16) int8_t vt[kAttnXTile][kAttnHeadDim];
    float s[kAttnXMaxSeq];
};

__global__ void __launch_bounds__(kAttnXThreads) k_attention_exact(AttnArgs a, ExactTabs ex, float inv_sqrt_d) {
    __shared__ AttnXSmem S;
    constexpr int hd = kAttnHeadDim;
    const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int groups = a.n_heads / a.n_kv > 0 ? a.n_heads / a.n_kv : 1;
    const int g = h / groups;
    const int half = a.rot / 2;
    grid_dependency_wait();
    grid_launch_dependents();
    const int pos = a.st->pos;
    if (pos < 0 || pos >= a.max_seq || pos >= kAttnXMaxSeq) return;
    const int q_dim = a.n_heads * hd, kv_dim = a.n_kv * hd;

    // ---- RoPE of q and k, int8 quantization of this position's k and v ----
    float kval = 0.f, vval = 0.f;
    if (tid < hd) {
        const float* qh = a.qkv + h * hd;
        const float* kh = a.qkv + q_dim + g * hd;
        float qv = qh[tid], kv = kh[tid];
        if (tid < 2 * half) {
            const int i = tid < half ? tid : tid - half;
            const float rc = a.cos_t[static_cast<long long>(pos) * half + i];
            const float rs = a.sin_t[static_cast<long long>(pos) * half + i];
            if (tid < half) {
                qv = __fmaf_rn(qv, rc, -__fmul_rn(qh[tid + half], rs));
                kv = __fmaf_rn(kv, rc, -__fmul_rn(kh[tid + half], rs));
            } else {
                qv = __fmaf_rn(qh[i], rs, __fmul_rn(qv, rc));
                kv = __fmaf_rn(kh[i], rs, __fmul_rn(kv, rc));
            }
        }
        S.q[tid] = qv;
        kval = kv;
        vval = a.qkv[q_dim + kv_dim + g * hd + tid];
    }
    {
        const float km = warp_max(fabsf(kval));
        const float vm = warp_max(fabsf(vval));
        if (tid < hd && lane == 0) {
            S.red[0][tid >> 6][(tid >> 5) & 1] = km;
            S.red[1][tid >> 6][(tid >> 5) & 1] = vm;
        }
    }
    __syncthreads();
    if (tid < hd) {
        const int b = tid >> 6;
        const float ka = fmaxf(S.red[0][b][0], S.red[0][b][1]);
        const float va = fmaxf(S.red[1][b][0], S.red[1][b][1]);
        const float ksc = ka > 1e-12f ? __fmul_rn(ka, inv127f()) : 1e-12f;
        const float vsc = va > 1e-12f ? __fmul_rn(va, inv127f()) : 1e-12f;
        int qk = __float2int_rn(__fmul_rn(kval, kv_code_inv(ka)));
        int qv = __float2int_rn(__fmul_rn(vval, kv_code_inv(va)));
        qk = qk < -127 ? -127 : (qk > 127 ? 127 : qk);
        qv = qv < -127 ? -127 : (qv > 127 ? 127 : qv);
        S.k[tid] = __fmul_rn(static_cast<float>(qk), ksc);
        S.v[tid] = __fmul_rn(static_cast<float>(qv), vsc);
        if (h % groups == 0) {
            const long long kb = (static_cast<long long>(pos) * a.n_kv + g) * hd;
            a.kq[kb + tid] = static_cast<int8_t>(qk);
            a.vq[kb + tid] = static_cast<int8_t>(qv);
            if ((tid & 63) == 0) {
                const long long sb = (static_cast<long long>(pos) * a.n_kv + g) * 2 + b;
                a.ks[sb] = ksc;
                a.vs[sb] = vsc;
            }
        }
    }
    __syncthreads();

    // ---- scores: one thread per position ----
    for (int p = tid; p <= pos; p += kAttnXThreads) {
        float dot = 0.0f;
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            float ln[8];
            if (p == pos) {
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int l = 0; l < 8; ++l) {
                        const int d = b * 64 + i * 8 + l;
                        ln[l] = __fmaf_rn(S.q[d], S.k[d], i == 0 ? 0.0f : ln[l]);
                    }
            } else {
                const long long rb = (static_cast<long long>(p) * a.n_kv + g) * hd + b * 64;
                const float sc = a.ks[(static_cast<long long>(p) * a.n_kv + g) * 2 + b];
                const uint4* kp = reinterpret_cast<const uint4*>(a.kq + rb);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint4 w4 = kp[c];
                    const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const int i = c * 2 + (e >> 3), l = e & 7;
                        const int code = static_cast<int8_t>((ww[e >> 2] >> (8 * (e & 3))) & 0xFFu);
                        const float kf = __fmul_rn(static_cast<float>(code), sc);
                        ln[l] = __fmaf_rn(S.q[b * 64 + i * 8 + l], kf, i == 0 ? 0.0f : ln[l]);
                    }
                }
            }
            const float hs = __fadd_rn(__fadd_rn(__fadd_rn(ln[0], ln[4]), __fadd_rn(ln[1], ln[5])),
                                       __fadd_rn(__fadd_rn(ln[2], ln[6]), __fadd_rn(ln[3], ln[7])));
            dot = __fadd_rn(dot, hs);
        }
        S.s[p] = __fmul_rn(dot, inv_sqrt_d);
    }
    __syncthreads();

    // ---- 64-position tiles in order ----
    float m = -INFINITY, l = 0.0f, num = 0.0f;
    for (int tk = 0; tk <= pos; tk += kAttnXTile) {
        const int span = min(kAttnXTile, pos + 1 - tk);
        // tile maximum (every thread computes it from shared memory: no broadcast)
        float tmax = -INFINITY;
        for (int p = 0; p < span; ++p) {
            const float sp = S.s[tk + p];
            tmax = (tmax < sp) ? sp : tmax;
        }
        const float nm = (m < tmax) ? tmax : m;
        const float old = (l > 0.0f) ? exact_expf(__fsub_rn(m, nm), ex) : 0.0f;
        if (tid < span) S.w[tid] = exact_expf(__fsub_rn(S.s[tk + tid], nm), ex);
        // stage the tile's V codes (16-byte pieces) and scales; this position's v comes from S.v
        for (int i = tid; i < span * (hd / 16); i += kAttnXThreads) {
            const int p = i / (hd / 16), c = i % (hd / 16);
            if (tk + p != pos)
                *reinterpret_cast<uint4*>(&S.vt[p][c * 16]) = *reinterpret_cast<const uint4*>(
                    a.vq + (static_cast<long long>(tk + p) * a.n_kv + g) * hd + c * 16);
        }
        for (int i = tid; i < span * 2; i += kAttnXThreads) {
            const int p = i >> 1, b = i & 1;
            if (tk + p != pos) S.vs[p][b] = a.vs[(static_cast<long long>(tk + p) * a.n_kv + g) * 2 + b];
        }
        __syncthreads();
        float tl = 0.0f, tn = 0.0f;
        for (int p = 0; p < span; ++p) {
            const float wp = S.w[p];
            tl = __fadd_rn(tl, wp);
            if (tid < hd) {
                const float vf = (tk + p == pos) ? S.v[tid]
                                                 : __fmul_rn(static_cast<float>(S.vt[p][tid]), S.vs[p][tid >> 6]);
                tn = __fmaf_rn(wp, vf, tn);
            }
        }
        l = __fadd_rn(__fmul_rn(l, old), tl);
        num = __fmaf_rn(num, old, tn);
        m = nm;
        __syncthreads();  // w / vt are rewritten by the next tile
    }
    if (tid < hd) a.out[h * hd + tid] = __fmul_rn(num, __fdiv_rn(1.0f, l));
    (void)warp;
}

}  // namespace asdsl
