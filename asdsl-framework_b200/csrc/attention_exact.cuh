// attention_exact.cuh -- the decode attention of one layer in the reference's compiled order
// (reference-exact numerics mode).
//
// Reference: rope_apply_inplace (unified_engine.cpp:768-801), set_kv_cache (:859-920) and
// compute_attention_flash_q8 (:922-1027).  Per query head, the reference computes:
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
// A tile's (tile_l, tile_num) depend only on the running maximum through that tile, so this
// kernel (one CTA per query head) computes every score, the running maxima (a short sequential
// scan over tiles), every weight, and all tiles' sums in parallel; only the final merge over
// tiles runs in order.  The cached K/V of earlier positions (up to kAttnXPrefetch of them) are
// copied into shared memory before the dependency wait, overlapping the qkv GEMV.
#pragma once

#include "engine_ops.cuh"
#include "exact_math.cuh"
#include "gemv_stream.cuh"  // the optional per-CTA timeline (tl_slot / tl_put)

namespace asdsl {

constexpr int kAttnXThreads = 256;
constexpr int kAttnXMaxSeq = 4096;
constexpr int kAttnXTile = 64;
constexpr int kAttnXPrefetch = 256;   // positions of cached K/V staged in shared memory
constexpr int kAttnXRow = kAttnHeadDim + 16;  // padded K row (conflict-free 16-byte loads per thread)

struct AttnXLayout {
    uint32_t s, w, tile, tn, kc, vc, ksc, vsc, total;
};

// shared-memory layout of one head for a cache of max_seq positions (bytes, 16-aligned pieces)
__host__ __device__ inline AttnXLayout attn_x_layout(int max_seq) {
    const uint32_t nt = static_cast<uint32_t>((max_seq + kAttnXTile - 1) / kAttnXTile);
    const uint32_t np = static_cast<uint32_t>(max_seq < kAttnXPrefetch ? max_seq : kAttnXPrefetch);
    AttnXLayout L;
    uint32_t o = 0;
    auto take = [&](uint32_t bytes) {
        const uint32_t at = o;
        o += (bytes + 15u) & ~15u;
        return at;
    };
    L.s = take(4u * max_seq);
    L.w = take(4u * max_seq);
    L.tile = take(4u * 4u * nt);  // per tile: running max, old scale, tile_l, tile max
    L.tn = take(4u * nt * kAttnHeadDim);
    L.kc = take(np * kAttnXRow);
    L.vc = take(np * kAttnHeadDim);
    L.ksc = take(8u * np);
    L.vsc = take(8u * np);
    L.total = o;
    return L;
}

__global__ void __launch_bounds__(kAttnXThreads) k_attention_exact(AttnArgs a, ExactTabs ex, float inv_sqrt_d) {
    extern __shared__ __align__(16) uint8_t dsm[];
    __shared__ float q_s[kAttnHeadDim], k_s[kAttnHeadDim], v_s[kAttnHeadDim];
    __shared__ float red[2][2][2];
    constexpr int hd = kAttnHeadDim;
    const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int groups = a.n_heads / a.n_kv > 0 ? a.n_heads / a.n_kv : 1;
    const int g = h / groups;
    const int half = a.rot / 2;
    const AttnXLayout L = attn_x_layout(a.max_seq);
    float* s_s = reinterpret_cast<float*>(dsm + L.s);
    float* w_s = reinterpret_cast<float*>(dsm + L.w);
    float* tile_s = reinterpret_cast<float*>(dsm + L.tile);  // [nt][4]: m_t, old_t, tl_t, tmax_t
    float* tn_s = reinterpret_cast<float*>(dsm + L.tn);
    int8_t* kc_s = reinterpret_cast<int8_t*>(dsm + L.kc);
    int8_t* vc_s = reinterpret_cast<int8_t*>(dsm + L.vc);
    float* ksc_s = reinterpret_cast<float*>(dsm + L.ksc);
    float* vsc_s = reinterpret_cast<float*>(dsm + L.vsc);

    // optional timeline records (template code 15 = this kernel; phases 11..15 below)
    __shared__ uint32_t s_tl;
    if constexpr (kTimeline) {
        if (tid == 0) s_tl = tl_slot();
        __syncthreads();
    }
    const TlCtx tlc{kTimeline ? s_tl : ~0u, 15u << 4, 0xFFFF0000u};
    if (tid == 0) tl_put(tlc, kTlStart);
    // the position is final here: the embedding kernel of this step ran to completion first
    const int pos = a.st->pos;
    const bool ok = pos >= 0 && pos < a.max_seq && pos < kAttnXMaxSeq;
    // ---- cached K/V of earlier positions -> shared memory (independent of the qkv kernel) ----
    const int np = ok ? min(pos, kAttnXPrefetch) : 0;
    for (int i = tid; i < np * 16; i += kAttnXThreads) {
        const int p = i >> 4, c = i & 15;  // 16 pieces of 16 bytes: 8 of K, 8 of V
        const long long rb = (static_cast<long long>(p) * a.n_kv + g) * hd;
        if (c < 8)
            *reinterpret_cast<uint4*>(kc_s + p * kAttnXRow + c * 16) =
                *reinterpret_cast<const uint4*>(a.kq + rb + c * 16);
        else
            *reinterpret_cast<uint4*>(vc_s + p * hd + (c - 8) * 16) =
                *reinterpret_cast<const uint4*>(a.vq + rb + (c - 8) * 16);
    }
    for (int i = tid; i < np * 2; i += kAttnXThreads) {
        const int p = i >> 1, b = i & 1;
        const long long sb = (static_cast<long long>(p) * a.n_kv + g) * 2 + b;
        ksc_s[2 * p + b] = a.ks[sb];
        vsc_s[2 * p + b] = a.vs[sb];
    }
    grid_dependency_wait();
    grid_launch_dependents();
    if (tid == 0) tl_put(tlc, kTlWaited);
    if (!ok) return;
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
        q_s[tid] = qv;
        kval = kv;
        vval = a.qkv[q_dim + kv_dim + g * hd + tid];
    }
    {
        const float km = warp_max(fabsf(kval));
        const float vm = warp_max(fabsf(vval));
        if (tid < hd && lane == 0) {
            red[0][tid >> 6][(tid >> 5) & 1] = km;
            red[1][tid >> 6][(tid >> 5) & 1] = vm;
        }
    }
    __syncthreads();
    if (tid < hd) {
        const int b = tid >> 6;
        const float ka = fmaxf(red[0][b][0], red[0][b][1]);
        const float va = fmaxf(red[1][b][0], red[1][b][1]);
        const float ksc = ka > 1e-12f ? __fmul_rn(ka, inv127f()) : 1e-12f;
        const float vsc = va > 1e-12f ? __fmul_rn(va, inv127f()) : 1e-12f;
        int qk = __float2int_rn(__fmul_rn(kval, kv_code_inv(ka)));
        int qv = __float2int_rn(__fmul_rn(vval, kv_code_inv(va)));
        qk = qk < -127 ? -127 : (qk > 127 ? 127 : qk);
        qv = qv < -127 ? -127 : (qv > 127 ? 127 : qv);
        k_s[tid] = __fmul_rn(static_cast<float>(qk), ksc);
        v_s[tid] = __fmul_rn(static_cast<float>(qv), vsc);
        if (pos < kAttnXPrefetch) {
            // this position's codes and scales join the staged rows: code * scale there is the
            // same product as k_s / v_s, so the loops below need no case for it
            kc_s[pos * kAttnXRow + tid] = static_cast<int8_t>(qk);
            vc_s[pos * hd + tid] = static_cast<int8_t>(qv);
            if ((tid & 63) == 0) {
                ksc_s[2 * pos + b] = ksc;
                vsc_s[2 * pos + b] = vsc;
            }
        }
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
    if (tid == 0) tl_put(tlc, kTlAttnRope);

    // ---- scores ----
    // short caches (every row staged, one pass): 8 threads per position, thread l running dot
    // lane l of both 64-dim blocks (the FMA chains below), folded by shuffles in the same order;
    // longer ones: one thread per position, its eight lanes in registers
    constexpr int kScoreGroupMaxPos = kAttnXThreads / 8 - 1;
    if (pos <= kScoreGroupMaxPos) {
        const int l = tid & 7;
        const unsigned m = 0xFFu << (tid & 24);  // this group of 8 lanes (one position)
        for (int p = tid >> 3; p <= pos; p += kAttnXThreads / 8) {
            const float sc0 = ksc_s[2 * p], sc1 = ksc_s[2 * p + 1];
            const int8_t* kr = kc_s + p * kAttnXRow + l;
            float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                acc0 = __fmaf_rn(q_s[i * 8 + l], __fmul_rn(small_int_to_float(kr[i * 8]), sc0), i == 0 ? 0.0f : acc0);
                acc1 = __fmaf_rn(q_s[64 + i * 8 + l], __fmul_rn(small_int_to_float(kr[64 + i * 8]), sc1),
                                 i == 0 ? 0.0f : acc1);
            }
            float a0 = __fadd_rn(acc0, __shfl_xor_sync(m, acc0, 4));  // l < 4: v_l + v_{l+4}
            float a1 = __fadd_rn(acc1, __shfl_xor_sync(m, acc1, 4));
            a0 = __fadd_rn(a0, __shfl_xor_sync(m, a0, 1));  // (a0 + a1), (a2 + a3)
            a1 = __fadd_rn(a1, __shfl_xor_sync(m, a1, 1));
            a0 = __fadd_rn(a0, __shfl_xor_sync(m, a0, 2));  // (a0 + a1) + (a2 + a3)
            a1 = __fadd_rn(a1, __shfl_xor_sync(m, a1, 2));
            if (l == 0) s_s[p] = __fmul_rn(__fadd_rn(__fadd_rn(0.0f, a0), a1), inv_sqrt_d);
        }
    }
    for (int p = (pos <= kScoreGroupMaxPos) ? pos + 1 : tid; p <= pos; p += kAttnXThreads) {
        float dot = 0.0f;
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            float ln[8];
            if (p == pos && pos >= kAttnXPrefetch) {
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int l = 0; l < 8; ++l) {
                        const int d = b * 64 + i * 8 + l;
                        ln[l] = __fmaf_rn(q_s[d], k_s[d], i == 0 ? 0.0f : ln[l]);
                    }
            } else {
                const bool staged = p < kAttnXPrefetch;
                const float sc = staged ? ksc_s[2 * p + b] : a.ks[(static_cast<long long>(p) * a.n_kv + g) * 2 + b];
                const int8_t* kr = staged ? kc_s + p * kAttnXRow + b * 64
                                          : a.kq + (static_cast<long long>(p) * a.n_kv + g) * hd + b * 64;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint4 w4 = *reinterpret_cast<const uint4*>(kr + c * 16);
                    const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const int i = c * 2 + (e >> 3), l = e & 7;
                        const int code = static_cast<int8_t>((ww[e >> 2] >> (8 * (e & 3))) & 0xFFu);
                        const float kf = __fmul_rn(static_cast<float>(code), sc);
                        ln[l] = __fmaf_rn(q_s[b * 64 + i * 8 + l], kf, i == 0 ? 0.0f : ln[l]);
                    }
                }
            }
            const float hs = __fadd_rn(__fadd_rn(__fadd_rn(ln[0], ln[4]), __fadd_rn(ln[1], ln[5])),
                                       __fadd_rn(__fadd_rn(ln[2], ln[6]), __fadd_rn(ln[3], ln[7])));
            dot = __fadd_rn(dot, hs);
        }
        s_s[p] = __fmul_rn(dot, inv_sqrt_d);
    }
    __syncthreads();
    if (tid == 0) tl_put(tlc, kTlAttnScores);

    // ---- tile maxima (one warp per tile), then the running maxima and old scales in order ----
    const int nt = (pos + kAttnXTile) / kAttnXTile;  // tiles covering positions 0..pos
    for (int t = warp; t < nt; t += kAttnXThreads / 32) {
        const int tk = t * kAttnXTile, span = min(kAttnXTile, pos + 1 - tk);
        float v = -INFINITY;
        if (lane < span) v = s_s[tk + lane];
        if (lane + 32 < span) {
            const float v2 = s_s[tk + lane + 32];
            v = (v < v2) ? v2 : v;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float u = __shfl_xor_sync(0xffffffffu, v, o);
            v = (v < u) ? u : v;
        }
        if (v == 0.0f) {
            // a zero maximum: +0 and -0 compare equal, so take the sequential first-maximum rule
            // (std::max keeps the earlier of equal values) to get its sign right
            float q = -INFINITY;
            for (int p = 0; p < span; ++p) {
                const float sp = s_s[tk + p];
                q = (q < sp) ? sp : q;
            }
            v = q;
        }
        if (lane == 0) tile_s[4 * t + 3] = v;
    }
    __syncthreads();
    if (tid == 0) {
        float m = -INFINITY;
        for (int t = 0; t < nt; ++t) {
            const float tm = tile_s[4 * t + 3];
            const float nm = (m < tm) ? tm : m;
            // after the first tile l > 0 (its maximum's weight is exp(0) = 1), so old is exp(m - nm)
            tile_s[4 * t + 1] = (t == 0) ? 0.0f : exact_expf(__fsub_rn(m, nm), ex);
            tile_s[4 * t + 0] = nm;
            m = nm;
        }
    }
    __syncthreads();
    if (tid == 0) tl_put(tlc, kTlAttnMaxima);
    // ---- weights of every position ----
    for (int p = tid; p <= pos; p += kAttnXThreads)
        w_s[p] = exact_expf(__fsub_rn(s_s[p], tile_s[4 * (p / kAttnXTile)]), ex);
    __syncthreads();
    if (tid == 0) tl_put(tlc, kTlAttnWeights);
    // ---- every tile's tile_l and tile_num (thread per (tile, dim)), in position order ----
    for (int i = tid; i < nt * hd; i += kAttnXThreads) {
        const int t = i / hd, d = i % hd;
        const int tk = t * kAttnXTile, span = min(kAttnXTile, pos + 1 - tk);
        float tl = 0.0f, tn = 0.0f;
        if (tk + span <= kAttnXPrefetch) {
            // every position of the tile is staged: one uniform loop whose loads run ahead of
            // the two sequential sums
            const int8_t* vr = vc_s + tk * hd + d;
            const float* sr = vsc_s + 2 * tk + (d >> 6);
            const float* wr = w_s + tk;
            int pp = 0;
            for (; pp + 8 <= span; pp += 8) {
                // eight positions' operands first, then the two sums in position order
                float wv[8], vv[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    wv[u] = wr[pp + u];
                    vv[u] = __fmul_rn(small_int_to_float(vr[(pp + u) * hd]), sr[2 * (pp + u)]);
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    tl = __fadd_rn(tl, wv[u]);
                    tn = __fmaf_rn(wv[u], vv[u], tn);
                }
            }
            for (; pp < span; ++pp) {
                const float wp = wr[pp];
                tl = __fadd_rn(tl, wp);
                tn = __fmaf_rn(wp, __fmul_rn(small_int_to_float(vr[pp * hd]), sr[2 * pp]), tn);
            }
            tn_s[t * hd + d] = tn;
            if (d == 0) tile_s[4 * t + 2] = tl;
            continue;
        }
        for (int pp = 0; pp < span; ++pp) {
            const int p = tk + pp;
            const float wp = w_s[p];
            tl = __fadd_rn(tl, wp);
            float vf;
            if (p == pos) {
                vf = v_s[d];
            } else if (p < kAttnXPrefetch) {
                vf = __fmul_rn(static_cast<float>(vc_s[p * hd + d]), vsc_s[2 * p + (d >> 6)]);
            } else {
                const long long rb = (static_cast<long long>(p) * a.n_kv + g) * hd;
                vf = __fmul_rn(static_cast<float>(a.vq[rb + d]), a.vs[(static_cast<long long>(p) * a.n_kv + g) * 2 + (d >> 6)]);
            }
            tn = __fmaf_rn(wp, vf, tn);
        }
        tn_s[t * hd + d] = tn;
        if (d == 0) tile_s[4 * t + 2] = tl;
    }
    __syncthreads();
    if (tid == 0) tl_put(tlc, kTlAttnSums);
    // ---- merge the tiles in order ----
    if (tid < hd) {
        float l = 0.0f, num = 0.0f;
        for (int t = 0; t < nt; ++t) {
            const float old = tile_s[4 * t + 1];
            l = __fadd_rn(__fmul_rn(l, old), tile_s[4 * t + 2]);
            num = __fmaf_rn(num, old, tn_s[t * hd + tid]);
        }
        a.out[h * hd + tid] = __fmul_rn(num, __fdiv_rn(1.0f, l));
    }
    if (tid == 0) tl_put(tlc, kTlEnd);
}

// ---------------------------------------------------------------------------
// Split form for long caches: the same operations, spread over (head, 128-position chunk) CTAs
// in two kernels, so every value -- score, tile maximum, running maximum, old scale, weight,
// tile sum -- is computed by the same expression as in k_attention_exact, and the merge over
// tiles runs in tile order as there: the outputs are bitwise the single-CTA kernel's.
//   k_attention_exact_scores: RoPE + this position's KV quantization (the chunk holding `pos`
//     stores it), the scores of the chunk's positions and its tiles' maxima -> global scratch;
//   k_attention_exact_sums: the running maxima through the chunk's tiles (a scan over the tile
//     maxima), old scales, weights, every tile's (tile_l, tile_num) -> global scratch; the last
//     CTA of the head merges all tiles in order.
// ---------------------------------------------------------------------------
// positions per CTA (2 tiles); measured on B200, exact decode at positions 1920-1983: 1.92 ms/token
// against 2.00 with 256-position chunks (the tile sums of a CTA are its critical path)
constexpr int kAttnXChunk = 128;
constexpr int kAttnXChunkTiles = kAttnXChunk / kAttnXTile;
constexpr int kAttnXResStride = kAttnHeadDim + 4;      // per tile: old, tile_l, pad, pad, num[128]

struct AttnXSplit {
    float* s;            // [n_heads][max_seq] scores
    float* tmax;         // [n_heads][max_tiles] tile maxima
    float* tres;         // [n_heads][max_tiles][kAttnXResStride]
    unsigned int* cnt;   // [n_heads] arrival counters of the sums kernel (re-armed by its last CTA)
};

__global__ void __launch_bounds__(kAttnXThreads)
    k_attention_exact_scores(AttnArgs a, ExactTabs ex, float inv_sqrt_d, AttnXSplit sp) {
    __shared__ __align__(16) int8_t kc_s[kAttnXChunk * kAttnXRow];
    __shared__ float ksc_s[2 * kAttnXChunk];
    __shared__ float q_s[kAttnHeadDim], k_s[kAttnHeadDim];
    __shared__ float red[2][2][2];
    __shared__ float s_s[kAttnXChunk];
    constexpr int hd = kAttnHeadDim;
    const int h = blockIdx.x, c = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int groups = a.n_heads / a.n_kv > 0 ? a.n_heads / a.n_kv : 1;
    const int g = h / groups;
    const int half = a.rot / 2;
    const int pos = a.st->pos;
    const int p0 = c * kAttnXChunk;
    const bool live = pos >= 0 && pos < a.max_seq && p0 <= pos;
    const int p1 = live ? min(pos + 1, p0 + kAttnXChunk) : p0;  // positions [p0, p1)
    const bool owner = live && pos < p0 + kAttnXChunk;
    // cached K of this chunk's earlier positions -> shared memory (independent of the qkv kernel)
    const int ncached = live ? (owner ? pos - p0 : p1 - p0) : 0;
    for (int i = tid; i < ncached * 8; i += kAttnXThreads) {
        const int pp = i >> 3, cc = i & 7;
        const long long rb = (static_cast<long long>(p0 + pp) * a.n_kv + g) * hd;
        *reinterpret_cast<uint4*>(kc_s + pp * kAttnXRow + cc * 16) = *reinterpret_cast<const uint4*>(a.kq + rb + cc * 16);
    }
    for (int i = tid; i < ncached * 2; i += kAttnXThreads) {
        const int pp = i >> 1, b = i & 1;
        ksc_s[i] = a.ks[(static_cast<long long>(p0 + pp) * a.n_kv + g) * 2 + b];
    }
    grid_dependency_wait();
    grid_launch_dependents();
    if (!live) return;
    const int q_dim = a.n_heads * hd, kv_dim = a.n_kv * hd;
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
        q_s[tid] = qv;
        kval = kv;
        vval = a.qkv[q_dim + kv_dim + g * hd + tid];
    }
    if (owner) {
        const float km = warp_max(fabsf(kval));
        const float vm = warp_max(fabsf(vval));
        if (tid < hd && lane == 0) {
            red[0][tid >> 6][(tid >> 5) & 1] = km;
            red[1][tid >> 6][(tid >> 5) & 1] = vm;
        }
    }
    __syncthreads();
    if (owner && tid < hd) {
        const int b = tid >> 6;
        const float ka = fmaxf(red[0][b][0], red[0][b][1]);
        const float va = fmaxf(red[1][b][0], red[1][b][1]);
        const float ksc = ka > 1e-12f ? __fmul_rn(ka, inv127f()) : 1e-12f;
        const float vsc = va > 1e-12f ? __fmul_rn(va, inv127f()) : 1e-12f;
        int qk = __float2int_rn(__fmul_rn(kval, kv_code_inv(ka)));
        int qv = __float2int_rn(__fmul_rn(vval, kv_code_inv(va)));
        qk = qk < -127 ? -127 : (qk > 127 ? 127 : qk);
        qv = qv < -127 ? -127 : (qv > 127 ? 127 : qv);
        k_s[tid] = __fmul_rn(static_cast<float>(qk), ksc);
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
    // scores: one thread per position (k_attention_exact's expression)
    float* s_g = sp.s + static_cast<long long>(h) * a.max_seq;
    for (int p = p0 + tid; p < p1; p += kAttnXThreads) {
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
                        ln[l] = __fmaf_rn(q_s[d], k_s[d], i == 0 ? 0.0f : ln[l]);
                    }
            } else {
                const float sc = ksc_s[2 * (p - p0) + b];
                const int8_t* kr = kc_s + (p - p0) * kAttnXRow + b * 64;
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    const uint4 w4 = *reinterpret_cast<const uint4*>(kr + cc * 16);
                    const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const int i = cc * 2 + (e >> 3), l = e & 7;
                        const int code = static_cast<int8_t>((ww[e >> 2] >> (8 * (e & 3))) & 0xFFu);
                        const float kf = __fmul_rn(static_cast<float>(code), sc);
                        ln[l] = __fmaf_rn(q_s[b * 64 + i * 8 + l], kf, i == 0 ? 0.0f : ln[l]);
                    }
                }
            }
            const float hs = __fadd_rn(__fadd_rn(__fadd_rn(ln[0], ln[4]), __fadd_rn(ln[1], ln[5])),
                                       __fadd_rn(__fadd_rn(ln[2], ln[6]), __fadd_rn(ln[3], ln[7])));
            dot = __fadd_rn(dot, hs);
        }
        const float sv = __fmul_rn(dot, inv_sqrt_d);
        s_s[p - p0] = sv;
        s_g[p] = sv;
    }
    __syncthreads();
    // tile maxima of this chunk (one warp per tile; a zero maximum takes the sequential rule)
    const int t0 = p0 / kAttnXTile, nt_own = (p1 - p0 + kAttnXTile - 1) / kAttnXTile;
    for (int tt = warp; tt < nt_own; tt += kAttnXThreads / 32) {
        const int tk = tt * kAttnXTile, span = min(kAttnXTile, p1 - p0 - tk);
        float v = -INFINITY;
        if (lane < span) v = s_s[tk + lane];
        if (lane + 32 < span) {
            const float v2 = s_s[tk + lane + 32];
            v = (v < v2) ? v2 : v;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float u = __shfl_xor_sync(0xffffffffu, v, o);
            v = (v < u) ? u : v;
        }
        if (v == 0.0f) {
            float q = -INFINITY;
            for (int pp = 0; pp < span; ++pp) {
                const float spv = s_s[tk + pp];
                q = (q < spv) ? spv : q;
            }
            v = q;
        }
        if (lane == 0) sp.tmax[static_cast<long long>(h) * ((a.max_seq + kAttnXTile - 1) / kAttnXTile) + t0 + tt] = v;
    }
}

__global__ void __launch_bounds__(kAttnXThreads)
    k_attention_exact_sums(AttnArgs a, ExactTabs ex, AttnXSplit sp) {
    __shared__ __align__(16) int8_t vc_s[kAttnXChunk * kAttnHeadDim];
    __shared__ float vsc_s[2 * kAttnXChunk];
    __shared__ float w_s[kAttnXChunk];
    __shared__ float m_s[kAttnXChunkTiles], mp_s[kAttnXChunkTiles], old_s[kAttnXChunkTiles];
    __shared__ float tm_s[kAttnXMaxSeq / kAttnXTile];
    __shared__ int last_s;
    constexpr int hd = kAttnHeadDim;
    const int h = blockIdx.x, c = blockIdx.y, tid = threadIdx.x;
    const int groups = a.n_heads / a.n_kv > 0 ? a.n_heads / a.n_kv : 1;
    const int g = h / groups;
    const int max_tiles = (a.max_seq + kAttnXTile - 1) / kAttnXTile;
    // the position is final here (the previous token's step advanced it); the V of earlier
    // positions was stored by earlier steps, so it is staged before the dependency wait
    const int pos = a.st->pos;
    const bool ok = pos >= 0 && pos < a.max_seq;
    const int p0 = c * kAttnXChunk;
    const bool live = ok && p0 <= pos;
    const int p1 = live ? min(pos + 1, p0 + kAttnXChunk) : p0;
    const int nold = live ? min(pos, p1) - p0 : 0;  // positions of this chunk before `pos`
    auto stage_v = [&](int pp0, int pp1) {
        for (int i = tid + pp0 * 8; i < pp1 * 8; i += kAttnXThreads) {
            const int pp = i >> 3, cc = i & 7;
            const long long rb = (static_cast<long long>(p0 + pp) * a.n_kv + g) * hd;
            *reinterpret_cast<uint4*>(vc_s + pp * hd + cc * 16) = *reinterpret_cast<const uint4*>(a.vq + rb + cc * 16);
        }
        for (int i = tid + pp0 * 2; i < pp1 * 2; i += kAttnXThreads) {
            const int pp = i >> 1, b = i & 1;
            vsc_s[i] = a.vs[(static_cast<long long>(p0 + pp) * a.n_kv + g) * 2 + b];
        }
    };
    stage_v(0, nold);
    grid_dependency_wait();  // the scores kernel (and this position's KV write) completed
    grid_launch_dependents();
    if (!ok) return;  // no CTA arrives: the counter stays armed
    const int t0 = p0 / kAttnXTile, nt_own = (p1 - p0 + kAttnXTile - 1) / kAttnXTile;
    const float* tmax = sp.tmax + static_cast<long long>(h) * max_tiles;
    float* tres = sp.tres + static_cast<long long>(h) * max_tiles * kAttnXResStride;
    if (live) {
        stage_v(nold, p1 - p0);  // this position's V, stored by the scores kernel
        // the tile maxima up to this chunk's last tile, loaded in parallel
        for (int t = tid; t < t0 + nt_own; t += kAttnXThreads) tm_s[t] = __ldcg(tmax + t);
        __syncthreads();
        if (tid == 0) {
            // running maxima through this chunk's tiles, as the single-CTA scan
            float m = -INFINITY;
            for (int t = 0; t < t0 + nt_own; ++t) {
                const float tm = tm_s[t];
                const float nm = (m < tm) ? tm : m;
                if (t >= t0) {
                    mp_s[t - t0] = m;
                    m_s[t - t0] = nm;
                }
                m = nm;
            }
        }
        __syncthreads();
        // old scales of this chunk's tiles, one thread each
        if (tid < nt_own) old_s[tid] = (t0 + tid == 0) ? 0.0f : exact_expf(__fsub_rn(mp_s[tid], m_s[tid]), ex);
        const float* s_g = sp.s + static_cast<long long>(h) * a.max_seq;
        for (int p = p0 + tid; p < p1; p += kAttnXThreads)
            w_s[p - p0] = exact_expf(__fsub_rn(__ldcg(s_g + p), m_s[(p - p0) / kAttnXTile]), ex);
        __syncthreads();
        for (int i = tid; i < nt_own * hd; i += kAttnXThreads) {
            const int tt = i / hd, d = i % hd;
            const int tk = tt * kAttnXTile, span = min(kAttnXTile, p1 - p0 - tk);
            float tl = 0.0f, tn = 0.0f;
            int pp = 0;
            for (; pp + 8 <= span; pp += 8) {
                // eight positions' operands first, then the two sums in position order
                float wv[8], vv[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int q = tk + pp + u;
                    wv[u] = w_s[q];
                    vv[u] = __fmul_rn(small_int_to_float(vc_s[q * hd + d]), vsc_s[2 * q + (d >> 6)]);
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    tl = __fadd_rn(tl, wv[u]);
                    tn = __fmaf_rn(wv[u], vv[u], tn);
                }
            }
            for (; pp < span; ++pp) {
                const int q = tk + pp;
                const float wp = w_s[q];
                tl = __fadd_rn(tl, wp);
                tn = __fmaf_rn(wp, __fmul_rn(small_int_to_float(vc_s[q * hd + d]), vsc_s[2 * q + (d >> 6)]), tn);
            }
            float* r = tres + static_cast<long long>(t0 + tt) * kAttnXResStride;
            r[4 + d] = tn;
            if (d == 0) {
                r[0] = old_s[tt];
                r[1] = tl;
            }
        }
    }
    // arrive; the head's last CTA merges every tile in order
    __threadfence();
    __syncthreads();
    if (tid == 0) last_s = atomicAdd(sp.cnt + h, 1u) == gridDim.y - 1u;
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    const int nt = (pos + kAttnXTile) / kAttnXTile;
    if (tid < hd) {
        // the tiles' values are loaded eight at a time, then folded in tile order
        constexpr int B = 8;
        float l = 0.0f, num = 0.0f;
        for (int tb = 0; tb < nt; tb += B) {
            float ov[B], tlv[B], tnv[B];
#pragma unroll
            for (int k = 0; k < B; ++k) {
                if (tb + k < nt) {
                    const float* r = tres + static_cast<long long>(tb + k) * kAttnXResStride;
                    ov[k] = __ldcg(r);
                    tlv[k] = __ldcg(r + 1);
                    tnv[k] = __ldcg(r + 4 + tid);
                }
            }
#pragma unroll
            for (int k = 0; k < B; ++k) {
                if (tb + k < nt) {
                    l = __fadd_rn(__fmul_rn(l, ov[k]), tlv[k]);
                    num = __fmaf_rn(num, ov[k], tnv[k]);
                }
            }
        }
        a.out[h * hd + tid] = __fmul_rn(num, __fdiv_rn(1.0f, l));
    }
    if (tid == 0) sp.cnt[h] = 0u;
}

}  // namespace asdsl
