// engine_ops.cuh -- the non-GEMV kernels of the device-resident decode step.
//
// Reference: asdsl/kernels/native/unified_engine.cpp (UnifiedEngine).
//   embedding row (fp16/fp32 -> fp32)        load_embed_row_f32         :181-197
//   partial RoPE on q and k                  rope_apply_inplace         :768-801
//   int8 KV write, 64-element blocks         set_kv_cache               :859-920
//   single-query GQA attention, int8 KV      compute_attention_flash_q8 :922-1027
//   KV zero-fill from a position             zero_kv_from               :1263-1283
//   engine lm_head quantizers (g32 / g128)   UnifiedEngine ctor         :320-400, :411-461
// The position and the token sequence live in device memory (DecodeState, seq[]),
// so one captured CUDA graph serves every decode step.
#pragma once

#include "common.cuh"

namespace asdsl {

struct DecodeState {
    int pos;  // position of the token being forwarded; that token is seq[pos]
    int pad[3];
};

template <typename T>
__device__ __forceinline__ float load_as_float(const T* p);
template <>
__device__ __forceinline__ float load_as_float<uint16_t>(const uint16_t* p) {
    return half_bits_to_float(*p);
}
template <>
__device__ __forceinline__ float load_as_float<float>(const float* p) {
    return *p;
}

// resid = fp32(embedding[seq[pos]])  (load_embed_row_f32); the token was range-checked on the host
template <typename T>
__global__ void k_embed(const T* __restrict__ emb, float* __restrict__ resid, const DecodeState* st,
                        const int* seq, int H, int V, int max_seq) {
    grid_dependency_wait();
    grid_launch_dependents();
    const int p = st->pos;
    if (p < 0 || p >= max_seq) return;
    const int tok = seq[p];
    if (tok < 0 || tok >= V) return;
    const T* row = emb + static_cast<long long>(tok) * H;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x)
        resid[i] = load_as_float<T>(row + i);
}

// ---------------------------------------------------------------------------
// Attention for one decode position.  One CTA per query head, 8 warps; each
// 8-lane group of a warp takes one position at a time (16 head dims per lane).
//   * RoPE on the head's q and on its KV head's k (pairs (i, i + rot/2));
//   * the current position's k (roped) and v are quantized per 64-dim block
//     exactly as set_kv_cache does; the first query head of each KV group stores
//     them, every head uses the dequantized values for position `pos` directly;
//   * online softmax over positions (libm-accurate expf), groups merged in a
//     fixed order at the end.
// head_dim is 128 (two 64-dim KV scale blocks); the host checks it.
// ---------------------------------------------------------------------------
constexpr int kAttnWarps = 8;
constexpr int kAttnGroups = kAttnWarps * 4;  // 8-lane position groups per CTA
constexpr int kAttnHeadDim = 128;
constexpr int kAttnPrefetch = 4;  // position blocks of cached K/V loaded before the dependency wait
// positions per CTA of the split-KV decode attention; measured on B200 at positions 1920-1983
// (fast decode, ms/token): 64 -> 1.60, 128 -> 1.41, 256 -> 1.33, 512 -> 1.55
constexpr int kAttnChunk = 256;
constexpr int kAttnPartStride = kAttnHeadDim + 4;  // floats per (head, chunk) partial: M, L, pad, acc[128]

// set_kv_cache's code multiplier as the reference's compiled code computes it
// (unified_engine.cpp:885-887): GCC folds 1/(absmax * fl(1/127)) into 127/absmax; a block with
// absmax <= 1e-12 has scale 1e-12 and multiplier fl(1e12)
__device__ __forceinline__ float kv_code_inv(float absmax) {
    return absmax > 1e-12f ? __fdiv_rn(127.0f, absmax) : __int_as_float(0x5368D4A5);
}

struct AttnArgs {
    const float* qkv;     // [q_dim + 2 kv_dim] (q | k | v), this layer's projection output
    float* out;           // [q_dim]
    int8_t* kq;           // this layer's K codes  [max_seq][n_kv][128]
    int8_t* vq;           // this layer's V codes
    float* ks;            // this layer's K scales [max_seq][n_kv][2]
    float* vs;
    const float* cos_t;   // [max_seq][rot/2]
    const float* sin_t;
    const DecodeState* st;
    int n_heads, n_kv, rot, max_seq;
    // split-KV decode attention (k_attention_split): per (head, chunk) partials and per-head
    // arrival counters (re-armed by the last CTA of each head)
    float* part;
    unsigned int* cnt;
};

// shared memory of one attention head
struct AttnSmem {
    float q[kAttnHeadDim];
    float k[kAttnHeadDim];  // dequantized current-position k, v
    float v[kAttnHeadDim];
    float red[2][2][2];     // [k|v][64-block][warp of block]
    float m[kAttnGroups], l[kAttnGroups];
    float sc[kAttnGroups];  // merge: exp(m[k] - M) of each live group, 0 for an empty one
    float num[kAttnGroups][kAttnHeadDim];
    float M;                // split-KV: the CTA's maximum over its live groups
    int last;               // split-KV: this CTA merges the head's chunks
};

// no-op wait: the caller already ordered the head after the kernel that wrote qkv
struct NoWait {
    __device__ __forceinline__ void operator()() const {}
};

// Split-KV: the head's last CTA to arrive merges the chunks' partials in chunk order:
// M = max over live chunks, L = sum l_c e^(M_c - M), out = (sum acc_c e^(M_c - M)) / L.
template <typename Sync>
__device__ __forceinline__ void attention_merge_chunks(const AttnArgs& a, int h, AttnSmem& S, int tid, Sync sync) {
    constexpr int hd = kAttnHeadDim;
    const int nch = gridDim.y;
    __threadfence();
    sync();
    if (tid == 0) {
        const unsigned int prev = atomicAdd(a.cnt + h, 1u);
        S.last = prev == static_cast<unsigned int>(nch) - 1u;
    }
    sync();
    if (!S.last) return;
    __threadfence();
    const float* base = a.part + static_cast<long long>(h) * nch * kAttnPartStride;
    if (tid < hd) {
        float M = -INFINITY;
        for (int c = 0; c < nch; ++c)
            if (__ldcg(base + c * kAttnPartStride + 1) > 0.0f) M = fmaxf(M, __ldcg(base + c * kAttnPartStride));
        float L = 0.0f, acc = 0.0f;
        for (int c = 0; c < nch; ++c) {
            const float lc = __ldcg(base + c * kAttnPartStride + 1);
            if (lc > 0.0f) {
                const float sc = expf(__ldcg(base + c * kAttnPartStride) - M);
                L = __fmaf_rn(lc, sc, L);
                acc = __fmaf_rn(__ldcg(base + c * kAttnPartStride + 4 + tid), sc, acc);
            }
        }
        a.out[h * hd + tid] = __fmul_rn(acc, __fdiv_rn(1.0f, L));
    }
    if (tid == 0) a.cnt[h] = 0u;  // re-armed for the next launch
}

// One head of the decode attention, run by kAttnWarps warps (thread ids 0..255).  `sync` is
// the barrier of those warps; kCoherent reads qkv through L2 (it was written by other CTAs of
// the same persistent kernel).
//
// Everything that does not depend on the kernel that wrote qkv -- the position, the RoPE
// factors and the first block of cached K/V -- is loaded before `wait()` returns, so those loads
// overlap the previous kernel's tail.
//
// kBatch: one token of a batch at position `batch_pos`, whose K/V (and those of the batch's
// other tokens) k_kv_write_rows already stored; every position, its own included, is read from
// the cache.  A cached position dequantizes to exactly the values the single-token head keeps in
// shared memory for its own position, so both give bit-identical outputs.
//
// kSplit: split-KV decode -- this CTA covers positions [chunk * kAttnChunk, (chunk + 1) *
// kAttnChunk) of the head (the chunk that holds `pos` also quantizes and stores this position's
// K/V); it leaves its (max, denominator, numerator) partial in a.part, and the head's last CTA to
// arrive merges the chunks in chunk order.  A context inside the first chunk gives the unsplit
// head's bits.
template <bool kCoherent, typename Sync, typename Wait = NoWait, bool kBatch = false, bool kSplit = false>
__device__ __forceinline__ void attention_head(const AttnArgs& a, int h, AttnSmem& S, int tid, Sync sync,
                                               Wait wait = Wait(), int batch_pos = -1, int chunk = 0) {
    constexpr int hd = kAttnHeadDim;
    const int groups = a.n_heads / a.n_kv > 0 ? a.n_heads / a.n_kv : 1;
    const int g = h / groups;
    const int half = a.rot / 2;
    const int pos = kBatch ? batch_pos : a.st->pos;
    if (pos < 0 || pos >= a.max_seq) {
        wait();
        return;
    }
    // positions [c0, c1) of this CTA (all of them without kSplit)
    const int c0 = kSplit ? chunk * kAttnChunk : 0;
    const int c1 = kSplit ? min(pos + 1, c0 + kAttnChunk) : pos + 1;
    const bool owns_pos = !kSplit || (c0 <= pos && pos < c0 + kAttnChunk);
    const int lane = tid & 31, warp = tid >> 5;
    const int q_dim = a.n_heads * hd, kv_dim = a.n_kv * hd;
    auto ldq = [&](const float* p) -> float {
        if constexpr (kCoherent) return __ldcg(p);
        else return *p;
    };
    // RoPE factors of this thread's dim pair
    float rc = 0.f, rs = 0.f;
    if (tid < 2 * half) {
        const int i = tid < half ? tid : tid - half;
        rc = a.cos_t[static_cast<long long>(pos) * half + i];
        rs = a.sin_t[static_cast<long long>(pos) * half + i];
    }
    // the cached positions of this thread's 8-lane group in the first kAttnPrefetch position
    // blocks (earlier tokens wrote them)
    const int grp = warp * 4 + (lane >> 3);  // 0 .. kAttnGroups-1
    const int l8 = lane & 7;                 // dims 16*l8 .. 16*l8+15 (scale block l8 >> 2)
    uint4 pk[kAttnPrefetch], pv[kAttnPrefetch];
    float pks[kAttnPrefetch], pvs[kAttnPrefetch];
#pragma unroll
    for (int i = 0; i < kAttnPrefetch; ++i) {
        const int p = c0 + i * kAttnGroups + grp;
        pk[i] = pv[i] = make_uint4(0u, 0u, 0u, 0u);
        pks[i] = pvs[i] = 0.f;
        if ((kBatch ? p <= pos : p < pos) && p < c1) {
            const long long rb = (static_cast<long long>(p) * a.n_kv + g) * hd + l8 * 16;
            const long long sb = (static_cast<long long>(p) * a.n_kv + g) * 2 + (l8 >> 2);
            pk[i] = *reinterpret_cast<const uint4*>(a.kq + rb);
            pv[i] = *reinterpret_cast<const uint4*>(a.vq + rb);
            pks[i] = a.ks[sb];
            pvs[i] = a.vs[sb];
        }
    }
    wait();

    // --- RoPE on q and k: thread t < 128 owns dim t (rope_apply_inplace :768-801) ---
    float kval = 0.f, vval = 0.f;
    if (tid < hd) {
        const float* qh = a.qkv + h * hd;
        const float* kh = a.qkv + q_dim + g * hd;
        float qv = ldq(qh + tid), kv = ldq(kh + tid);
        if (tid < half) {
            // o0 = fma(x_first, c, -(x_second * s))
            qv = __fmaf_rn(qv, rc, -__fmul_rn(ldq(qh + tid + half), rs));
            kv = __fmaf_rn(kv, rc, -__fmul_rn(ldq(kh + tid + half), rs));
        } else if (tid < 2 * half) {
            // o1 = fma(x_first, s, x_second * c)
            const int i = tid - half;
            qv = __fmaf_rn(ldq(qh + i), rs, __fmul_rn(qv, rc));
            kv = __fmaf_rn(ldq(kh + i), rs, __fmul_rn(kv, rc));
        }
        S.q[tid] = qv;
        kval = kv;
        vval = ldq(a.qkv + q_dim + kv_dim + g * hd + tid);
    }
    // --- quantize this position's k and v per 64-dim block (set_kv_cache :872-917) ---
    // dims 0..63 are warps 0-1, dims 64..127 warps 2-3
    if constexpr (!kBatch) {
        const float km = warp_max(fabsf(kval));
        const float vm = warp_max(fabsf(vval));
        if (tid < hd && lane == 0) {
            S.red[0][tid >> 6][(tid >> 5) & 1] = km;
            S.red[1][tid >> 6][(tid >> 5) & 1] = vm;
        }
        sync();
        if (tid < hd) {
            // every thread derives its block's scales from the two warp maxima (no second barrier)
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
            if (h % groups == 0 && owns_pos) {
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
    }
    sync();

    // --- scores + online softmax: an 8-lane group per position, 16 dims per lane ---
    const float inv_sqrt_d = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(hd)));
    float qreg[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) qreg[i] = S.q[l8 * 16 + i];
    float m = -INFINITY, l = 0.0f;
    float num[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) num[i] = 0.0f;
    const int npos = c1;
    for (int p0 = c0; p0 < npos; p0 += kAttnGroups) {
        const int p = p0 + grp;
        const bool live = p < npos;  // uniform within the 8-lane group
        float dot = 0.0f;
        float vdq[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) vdq[i] = 0.0f;
        if (live) {
            if (!kBatch && p == pos) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    dot = __fmaf_rn(qreg[i], S.k[l8 * 16 + i], dot);
                    vdq[i] = S.v[l8 * 16 + i];
                }
            } else {
                uint4 kw = make_uint4(0u, 0u, 0u, 0u), vw = kw;
                float ksc = 0.f, vsc = 0.f;
                const int blk = (p0 - c0) / kAttnGroups;
#pragma unroll
                for (int i = 0; i < kAttnPrefetch; ++i)
                    if (blk == i) {
                        kw = pk[i];
                        vw = pv[i];
                        ksc = pks[i];
                        vsc = pvs[i];
                    }
                if (blk >= kAttnPrefetch) {
                    const long long rb = (static_cast<long long>(p) * a.n_kv + g) * hd + l8 * 16;
                    const long long sb = (static_cast<long long>(p) * a.n_kv + g) * 2 + (l8 >> 2);
                    kw = *reinterpret_cast<const uint4*>(a.kq + rb);
                    vw = *reinterpret_cast<const uint4*>(a.vq + rb);
                    ksc = a.ks[sb];
                    vsc = a.vs[sb];
                }
                const uint32_t kk[4] = {kw.x, kw.y, kw.z, kw.w};
                const uint32_t vv[4] = {vw.x, vw.y, vw.z, vw.w};
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int kc = static_cast<int8_t>((kk[i >> 2] >> (8 * (i & 3))) & 0xFF);
                    const int vc = static_cast<int8_t>((vv[i >> 2] >> (8 * (i & 3))) & 0xFF);
                    dot = __fmaf_rn(qreg[i], __fmul_rn(small_int_to_float(kc), ksc), dot);
                    vdq[i] = __fmul_rn(small_int_to_float(vc), vsc);
                }
            }
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        dot += __shfl_xor_sync(0xffffffffu, dot, 2);
        dot += __shfl_xor_sync(0xffffffffu, dot, 4);
        if (live) {
            const float s = __fmul_rn(dot, inv_sqrt_d);
            const float nm = fmaxf(m, s);
            const float old_scale = (l > 0.0f) ? expf(m - nm) : 0.0f;
            const float w = expf(s - nm);
            l = __fmaf_rn(l, old_scale, w);
#pragma unroll
            for (int i = 0; i < 16; ++i) num[i] = __fmaf_rn(w, vdq[i], __fmul_rn(num[i], old_scale));
            m = nm;
        }
    }
    if (l8 == 0) {
        S.m[grp] = m;
        S.l[grp] = l;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) S.num[grp][l8 * 16 + i] = num[i];
    sync();
    // --- merge the groups in a fixed order --------------------------------------------
    // warp 0: the maximum over live groups, each group's exp(m - M) once, and the denominator
    if (warp == 0) {
        static_assert(kAttnGroups == 32, "one lane per position group");
        const bool live_k = S.l[lane] > 0.0f;
        float M = live_k ? S.m[lane] : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        S.sc[lane] = live_k ? expf(S.m[lane] - M) : 0.0f;
        if (lane == 0) S.M = M;
    }
    sync();
    if (tid < hd) {
        float L = 0.0f, acc = 0.0f;
        for (int k = 0; k < kAttnGroups; ++k) {
            if (S.l[k] > 0.0f) {
                L = __fmaf_rn(S.l[k], S.sc[k], L);
                acc = __fmaf_rn(S.num[k][tid], S.sc[k], acc);
            }
        }
        if constexpr (!kSplit) {
            a.out[h * hd + tid] = __fmul_rn(acc, __fdiv_rn(1.0f, L));
        } else {
            float* pp = a.part + (static_cast<long long>(h) * gridDim.y + chunk) * kAttnPartStride;
            pp[4 + tid] = acc;
            if (tid == 0) {
                pp[0] = S.M;
                pp[1] = L;  // 0: no live position in this chunk
            }
        }
    }
    if constexpr (kSplit) attention_merge_chunks(a, h, S, tid, sync);
}

struct BlockSync {
    __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

// the programmatic-launch wait on the qkv kernel, taken inside the head after its independent loads
struct GridWait {
    __device__ __forceinline__ void operator()() const {
        grid_dependency_wait();
        grid_launch_dependents();
    }
};

__global__ void __launch_bounds__(kAttnWarps * 32) k_attention(AttnArgs a) {
    __shared__ AttnSmem S;
    attention_head<false>(a, blockIdx.x, S, threadIdx.x, BlockSync(), GridWait());
}

// split-KV decode attention: grid (n_heads, ceil(max_seq / kAttnChunk)); CTA (h, c) covers
// positions [c * kAttnChunk, (c + 1) * kAttnChunk) of head h, chunks past the position only
// arrive at the head's counter.  Replaces the serial position loop of one CTA per head at long
// contexts (unified_engine.cpp:922-1027, whose result this merge reproduces within the fp32
// reassociation of the chunk sums).
__global__ void __launch_bounds__(kAttnWarps * 32) k_attention_split(AttnArgs a) {
    __shared__ AttnSmem S;
    const int h = blockIdx.x, c = blockIdx.y;
    const int pos = a.st->pos;
    if (pos >= 0 && pos < a.max_seq && c * kAttnChunk > pos) {
        // no position of this chunk is live: leave an empty partial and arrive
        grid_dependency_wait();
        grid_launch_dependents();
        if (threadIdx.x == 0) a.part[(static_cast<long long>(h) * gridDim.y + c) * kAttnPartStride + 1] = 0.0f;
        attention_merge_chunks(a, h, S, threadIdx.x, BlockSync());
        return;
    }
    attention_head<false, BlockSync, GridWait, false, true>(a, h, S, threadIdx.x, BlockSync(), GridWait(), -1, c);
}

// ---------------------------------------------------------------------------
// Batched forward (n tokens at positions start .. start + n - 1, row t of every activation
// block belongs to token t).  The KV writes of all n tokens run first (k_kv_write_rows), then
// every (head, token) pair attends over the positions <= its own, all read from the cache.
// ---------------------------------------------------------------------------

// resid[t] = fp32(embedding[tok[t]]); the tokens were range-checked on the host
template <typename T>
__global__ void k_embed_rows(const T* __restrict__ emb, float* __restrict__ resid, const int* tok, int H) {
    const int t = blockIdx.y;
    const T* row = emb + static_cast<long long>(tok[t]) * H;
    float* dst = resid + static_cast<long long>(t) * H;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x)
        dst[i] = load_as_float<T>(row + i);
}

// RoPE on k, then the int8 KV write of one (KV head, token): the arithmetic of attention_head's
// single-token write (set_kv_cache :859-920), one thread per head dim (128 threads)
__global__ void __launch_bounds__(kAttnHeadDim) k_kv_write_rows(AttnArgs a, int start, int qkv_stride) {
    constexpr int hd = kAttnHeadDim;
    const int g = blockIdx.x, t = blockIdx.y;
    const int pos = start + t;
    if (pos < 0 || pos >= a.max_seq) return;
    const int tid = threadIdx.x, lane = tid & 31;
    const int half = a.rot / 2;
    const int q_dim = a.n_heads * hd, kv_dim = a.n_kv * hd;
    const float* row = a.qkv + static_cast<long long>(t) * qkv_stride;
    const float* kh = row + q_dim + g * hd;
    float kval = kh[tid];
    if (tid < 2 * half) {
        const int i = tid < half ? tid : tid - half;
        const float rc = a.cos_t[static_cast<long long>(pos) * half + i];
        const float rs = a.sin_t[static_cast<long long>(pos) * half + i];
        if (tid < half) kval = __fmaf_rn(kval, rc, -__fmul_rn(kh[tid + half], rs));
        else kval = __fmaf_rn(kh[i], rs, __fmul_rn(kval, rc));
    }
    const float vval = row[q_dim + kv_dim + g * hd + tid];
    __shared__ float red[2][2][2];  // [k|v][64-block][warp of block]
    const float km = warp_max(fabsf(kval));
    const float vm = warp_max(fabsf(vval));
    if (lane == 0) {
        red[0][tid >> 6][(tid >> 5) & 1] = km;
        red[1][tid >> 6][(tid >> 5) & 1] = vm;
    }
    __syncthreads();
    const int b = tid >> 6;
    const float ka = fmaxf(red[0][b][0], red[0][b][1]);
    const float va = fmaxf(red[1][b][0], red[1][b][1]);
    const float ksc = ka > 1e-12f ? __fmul_rn(ka, inv127f()) : 1e-12f;
    const float vsc = va > 1e-12f ? __fmul_rn(va, inv127f()) : 1e-12f;
    int qk = __float2int_rn(__fmul_rn(kval, kv_code_inv(ka)));
    int qv = __float2int_rn(__fmul_rn(vval, kv_code_inv(va)));
    qk = qk < -127 ? -127 : (qk > 127 ? 127 : qk);
    qv = qv < -127 ? -127 : (qv > 127 ? 127 : qv);
    const long long kb = (static_cast<long long>(pos) * a.n_kv + g) * hd;
    a.kq[kb + tid] = static_cast<int8_t>(qk);
    a.vq[kb + tid] = static_cast<int8_t>(qv);
    if ((tid & 63) == 0) {
        const long long sb = (static_cast<long long>(pos) * a.n_kv + g) * 2 + b;
        a.ks[sb] = ksc;
        a.vs[sb] = vsc;
    }
}

// attention of every (query head, token) pair of the batch: grid (n_heads, n)
__global__ void __launch_bounds__(kAttnWarps * 32) k_attention_rows(AttnArgs a, int start, int qkv_stride) {
    __shared__ AttnSmem S;
    const int t = blockIdx.y;
    AttnArgs at = a;
    at.qkv = a.qkv + static_cast<long long>(t) * qkv_stride;
    at.out = a.out + static_cast<long long>(t) * a.n_heads * kAttnHeadDim;
    attention_head<false, BlockSync, NoWait, true>(at, blockIdx.x, S, threadIdx.x, BlockSync(), NoWait(), start + t);
}

// decode step done: seq[pos + 1] = argmax token, pos += 1 (seq holds max_seq + 1 entries;
// a step at an out-of-range position forwarded nothing and does not advance)
__global__ void k_advance_decode(DecodeState* st, int* seq, const int* argmax_idx, int max_seq) {
    grid_dependency_wait();
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const int p = st->pos;
    if (p < 0 || p >= max_seq) return;
    seq[p + 1] = *argmax_idx;
    st->pos = p + 1;
}

// prefill step done (no lm_head): pos += 1, the next token is already in seq
__global__ void k_advance_prefill(DecodeState* st, int max_seq) {
    grid_dependency_wait();
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const int p = st->pos;
    if (p < 0 || p >= max_seq) return;
    st->pos = p + 1;
}

// zero_kv_from: codes 0 and scales 1.0 for positions >= from in every layer
__global__ void k_kv_fill(int8_t* kq, int8_t* vq, float* ks, float* vs, int layers, long long per_layer_codes,
                          long long per_layer_scales, long long from_codes, long long from_scales) {
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    const long long t0 = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
    const long long nc = per_layer_codes - from_codes;
    const long long ns = per_layer_scales - from_scales;
    for (int l = 0; l < layers; ++l) {
        for (long long i = t0; i < nc; i += stride) {
            kq[l * per_layer_codes + from_codes + i] = 0;
            vq[l * per_layer_codes + from_codes + i] = 0;
        }
        for (long long i = t0; i < ns; i += stride) {
            ks[l * per_layer_scales + from_scales + i] = 1.0f;
            vs[l * per_layer_scales + from_scales + i] = 1.0f;
        }
    }
}

// ---------------------------------------------------------------------------
// engine lm_head quantizers, bit-exact with the reference constructor:
// one thread per (row, group); amax < 1e-12 -> scale 0, nibbles 0x88;
// else scale = fp16_rne(amax * fl(1/7)), q = clamp(round_half_away(x * (7/amax)) + 8, 0, 15)
// ---------------------------------------------------------------------------
// 8 codes of 4 bits, low nibble = even element, clamp(round_half_away(x * inv) + 8, 0, 15)
__device__ __forceinline__ uint32_t lm_pack8(const float* x, float inv) {
    uint32_t w = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        int q = static_cast<int>(roundf(__fmul_rn(x[j], inv))) + 8;
        q = q < 0 ? 0 : (q > 15 ? 15 : q);
        w |= static_cast<uint32_t>(q) << (4 * j);
    }
    return w;
}

// fp16 bits of amax * fl(1/7), or 0 for an all-zero group
__device__ __forceinline__ uint32_t lm_scale_bits(float amax) {
    if (amax < 1e-12f) return 0u;
    return static_cast<uint32_t>(__half_as_ushort(__float2half_rn(__fmul_rn(amax, inv7f()))));
}

template <typename T>
__global__ void k_lmhead_quant_preq2(const T* __restrict__ w, uint32_t* __restrict__ meta,
                                     uint4* __restrict__ quant, int rows, int cols) {
    const int ng = cols / 32;
    const long long total = static_cast<long long>(rows) * ng;
    for (long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = t / ng;
        const int g = static_cast<int>(t - r * ng);
        const T* src = w + r * cols + g * 32;
        float x[32];
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            x[j] = load_as_float<T>(src + j);
            amax = fmaxf(amax, fabsf(x[j]));
        }
        // meta word: fp16 scale (low half), fp16 zero 8.0 = 0x4800 (high half)
        meta[r * ng + g] = lm_scale_bits(amax) | (0x4800u << 16);
        uint4 qv = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
        if (amax >= 1e-12f) {
            const float inv = __fdiv_rn(7.0f, amax);
            qv.x = lm_pack8(x, inv);
            qv.y = lm_pack8(x + 8, inv);
            qv.z = lm_pack8(x + 16, inv);
            qv.w = lm_pack8(x + 24, inv);
        }
        // preq2 band slot: [r/4][g][r%4][16 bytes]
        quant[((r >> 2) * ng + g) * 4 + (r & 3)] = qv;
    }
}

// g128 variant, written directly in the banded device layout
// (quant [nb][K/128][4][64], scales [nb][K/128][4] fp16)
template <typename T>
__global__ void k_lmhead_quant_q128b(const T* __restrict__ w, uint4* __restrict__ quant,
                                     uint16_t* __restrict__ scales, int rows, int cols) {
    const int ng = cols / 128;
    const long long total = static_cast<long long>(rows) * ng;
    for (long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = t / ng;
        const int g = static_cast<int>(t - r * ng);
        const T* src = w + r * cols + g * 128;
        float amax = 0.0f;
        for (int j = 0; j < 128; ++j) amax = fmaxf(amax, fabsf(load_as_float<T>(src + j)));
        const long long slot = ((r >> 2) * ng + g) * 4 + (r & 3);
        scales[slot] = static_cast<uint16_t>(lm_scale_bits(amax));
        const float inv = amax >= 1e-12f ? __fdiv_rn(7.0f, amax) : 0.0f;
        for (int c = 0; c < 4; ++c) {
            uint4 qv = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
            if (amax >= 1e-12f) {
                float x[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) x[j] = load_as_float<T>(src + c * 32 + j);
                qv.x = lm_pack8(x, inv);
                qv.y = lm_pack8(x + 8, inv);
                qv.z = lm_pack8(x + 16, inv);
                qv.w = lm_pack8(x + 24, inv);
            }
            quant[slot * 4 + c] = qv;
        }
    }
}

}  // namespace asdsl
