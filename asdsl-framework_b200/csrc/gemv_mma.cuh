// gemv_mma.cuh -- multi-token W4A8 GEMV on the tensor cores (8 or 16 activation rows).
//
// Same semantics as the multi-token path of k_stream_gemv (config 4, speculative
// verification: Y[t] = W . A8(X[t]) for every token t, each token's A8 quantized exactly as the
// single-token kernel does), but the per-group integer dots of 16 weight rows x 8 tokens come
// from one mma.sync.m16n8k32 (s8 x s8 -> s32) instead of 16 x 8 lane dp4a chains:
//
//   A (16 x 32): rows r and r+8 of a 16-row tile (four 4-row bands).  Lane (g = lane/4,
//     t = lane%4) holds 32-bit word t of the row's 16 nibble bytes of the group, expanded in
//     place: low nibbles (elements 8t+0,2,4,6) as the k-columns 4t..4t+3 and high nibbles
//     (8t+1,3,5,7) as the k-columns 16+4t..16+4t+3;
//   B (32 x 8): token g's A8 codes in the same k order -- words 2t and 2t+1 of the permuted
//     activation record the prologue already writes (e_t = x[8t], x[8t+2], ...; o_t = x[8t+1], ...);
//   C (16 x 8): the exact int32 group dots, then the reference's per-group combine in fp32
//     (preq/preq2: dot*(ws*xs) - (wz*ws)*xss; Q4_K: (sc*dot - m*xsum)*xs).
//
// Work item = (16-row tile, group of 8 tokens, K part); K parts of a tile are summed in shared
// memory in a fixed order by the last one to finish (deterministic).  The weights stream through
// the same producer / mbarrier ring as the single-token kernel (tile-aligned chunks).  Only the
// float summation order across groups differs from k single-token calls (within the 1e-3 bar).
#pragma once

#include "launch.cuh"

namespace asdsl {

__device__ __forceinline__ void mma_s8_m16n8k32(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                 uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int FMT>
struct MmaFmt {
    static constexpr bool kSupported = (FMT == kFmtPreq2 || FMT == kFmtPreq || FMT == kFmtQ4K);
};

// Byte addresses, inside a stage, of row `slot` of unit `u` (relative to the chunk): nibble word
// t of group q, and the group's scale bits (preq / preq2: fp16 scale | fp16 zero << 16; Q4_K:
// the super-block address).
template <int FMT>
struct MmaRow {
    uint32_t nib;   // address of nibble word t of group q0
    uint32_t meta;  // preq2 / preq: address of the 4 scale bytes of group q0; Q4_K: row base
    __device__ __forceinline__ void init(uint32_t ub0, uint32_t ub1, int nq, int row_bytes, int unit, int slot,
                                         int t, int q0) {
        if constexpr (FMT == kFmtPreq2) {
            // quant band: [ng][4 rows][16 B]; meta band: [4 rows][ng][4 B]
            nib = ub0 + static_cast<uint32_t>(unit * nq * 64 + q0 * 64 + slot * 16 + t * 4);
            meta = ub1 + static_cast<uint32_t>(unit * nq * 16 + slot * nq * 4 + q0 * 4);
        } else if constexpr (FMT == kFmtPreq) {
            // row-major 20-byte blocks: scale, zero, 16 nibble bytes
            const uint32_t row = ub0 + static_cast<uint32_t>((unit * 4 + slot) * row_bytes);
            nib = row + static_cast<uint32_t>(q0 * 20 + 4 + t * 4);
            meta = row + static_cast<uint32_t>(q0 * 20);
        } else {
            // row-major 144-byte super-blocks: d, dmin, 12 bytes of 6-bit scales, 8 x 16 nibble bytes
            meta = ub0 + static_cast<uint32_t>((unit * 4 + slot) * row_bytes);
            nib = meta + static_cast<uint32_t>(t * 4);
        }
    }
    // nibble word / scale bits of group q = q0 + dq
    __device__ __forceinline__ uint32_t word_at(int q, uint32_t dq) const {
        if constexpr (FMT == kFmtPreq2) return lds32(nib + dq * 64u);
        else if constexpr (FMT == kFmtPreq) return lds32(nib + dq * 20u);
        else return lds32(nib + static_cast<uint32_t>((q >> 3) * 144 + 16 + (q & 7) * 16));
    }
    __device__ __forceinline__ uint32_t meta_at(uint32_t dq) const {
        if constexpr (FMT == kFmtPreq2) return lds32(meta + dq * 4u);
        else return lds32(meta + dq * 20u);
    }
    __device__ __forceinline__ uint32_t word(int q) const {
        if constexpr (FMT == kFmtQ4K)
            return lds32(nib + static_cast<uint32_t>((q >> 3) * 144 + 16 + (q & 7) * 16));
        else
            return lds32(nib);
    }
    __device__ __forceinline__ void advance() {
        if constexpr (FMT == kFmtPreq2) {
            nib += 64;
            meta += 4;
        } else if constexpr (FMT == kFmtPreq) {
            nib += 20;
            meta += 20;
        }
    }
    // fp32 factors of this row's group q: preq / preq2 (ws*1, wz*ws); Q4_K (d*sc, dmin*m)
    __device__ __forceinline__ float2 factors(int q) const {
        if constexpr (FMT == kFmtQ4K) {
            const uint32_t blk = meta + static_cast<uint32_t>((q >> 3) * 144);
            const uint32_t dd = lds32(blk);
            const uint32_t sb = static_cast<uint32_t>(q & 7);
            auto get6 = [&](uint32_t idx) -> int {
                const uint32_t bit = idx * 6u, byte = bit >> 3, off = bit & 7u;
                const uint32_t lo = lds8(blk + 4u + byte);
                if (off <= 2) return static_cast<int>((lo >> off) & 0x3Fu);
                return static_cast<int>(((lo >> off) | (lds8(blk + 5u + byte) << (8u - off))) & 0x3Fu);
            };
            return make_float2(__fmul_rn(half_bits_to_float(dd), static_cast<float>(get6(sb))),
                               __fmul_rn(half_bits_to_float(dd >> 16), static_cast<float>(get6(sb + 8u))));
        } else {
            const float2 sz = half2_bits_to_float2(lds32(meta));  // (scale, zero)
            return make_float2(sz.x, __fmul_rn(sz.y, sz.x));
        }
    }
};

// the nibble word of one row expanded into the two A registers of its k columns
__device__ __forceinline__ void expand_nibbles(uint32_t w, uint32_t& lo, uint32_t& hi) {
    lo = w & 0x0F0F0F0Fu;
    hi = (w >> 4) & 0x0F0F0F0Fu;
}

template <int FMT, int PRO, int NT>
__global__ void __launch_bounds__(kThreads, 1) k_stream_gemv_mma(const PipeArgs pa, const GemvArgs ga) {
    static_assert(NT == 8 || NT == 16, "tensor-core path for 8 or 16 tokens");
    static_assert(MmaFmt<FMT>::kSupported, "format without a tensor-core path");
    constexpr int NS = FmtTraits<FMT>::kStreams;
    constexpr int kOct = NT / 8;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    uint8_t* stages = smem + pa.stage_off;
    const int S = pa.n_stages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // tile-aligned unit range of this CTA (a tile = 4 units = 16 rows)
    const long long U = pa.n_units;
    const long long tiles = (U + 3) / 4;
    const long long t0 = tiles * blockIdx.x / gridDim.x;
    const long long t1 = tiles * (blockIdx.x + 1) / gridDim.x;
    const long long u0 = 4 * t0;
    const long long u1 = (4 * t1 < U) ? 4 * t1 : U;
    const int CU = pa.units_per_chunk;  // a multiple of 4
    const int TPC = CU / 4;             // tiles per chunk
    const int P = pa.k_parts;
    const int ntok = ga.n_tokens;
    const int n_oct = (ntok + 7) / 8;
    float* s_part = reinterpret_cast<float*>(smem + pa.split_off);    // [S][TPC][kOct][P][16 x 8]
    int* s_cnt = reinterpret_cast<int*>(s_part + S * TPC * kOct * P * 128);  // [S][TPC][kOct]

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_mbar_init();
    }
    if (P > 1)
        for (int i = threadIdx.x; i < S * TPC * kOct; i += blockDim.x) s_cnt[i] = 0;
    __syncthreads();
    grid_launch_dependents();

    if (warp == kProducerWarp) {
        if (lane != 0) return;
        const uint64_t pol = l2_policy_evict_first();
        int jg = 0;
        produce_chunks<NS, 1>(pa, u0, u1, stages, pa.stage_bytes, S, full, empty, jg, ga.status, pol);
        drain_ring(full, S, jg, ga.status);
        return;
    }

    grid_dependency_wait();
    const uint32_t xa_stride = xarea_layout_bytes(ga.K, ga.gs, false);
    token_prologue<PRO>(ga, smem + pa.xarea_off, xa_stride);

    const int K = ga.K;
    const int M = ga.M;
    const int nq = K >> 5;
    const int g = lane >> 2, tq = lane & 3;
    const uint32_t xbase = smem_u32(smem + pa.xarea_off);
    const uint32_t xs_off = (static_cast<uint32_t>(K) + 15u) & ~15u;  // x8[K] then xs[nq], xss[nq], xsi[nq]
    const uint32_t nq4 = 4u * static_cast<uint32_t>(nq);
    const int row_a = g, row_b = g + 8;  // tile rows of this lane's A / C elements
    const int n_items_per_tile = n_oct * P;

    int s = 0, use = 0;
    int item_base = 0;
    const uint32_t ring_s = smem_u32(stages);
    const int n_chunks = static_cast<int>((u1 - u0 + CU - 1) / CU);
    for (int j = 0; j < n_chunks; ++j) {
        if (!mbar_wait(&full[s], use & 1)) {
            if (lane == 0) atomicOr(ga.status, kStatusWaitFull);
            return;
        }
        const long long cb = u0 + static_cast<long long>(j) * CU;
        const int n_units_here = static_cast<int>(((cb + CU < u1) ? cb + CU : u1) - cb);
        const int tiles_here = (n_units_here + 3) / 4;
        const uint32_t st_s = ring_s + static_cast<uint32_t>(s) * pa.stage_bytes;
        uint32_t ub[NS];
#pragma unroll
        for (int i = 0; i < NS; ++i) ub[i] = st_s + pa.s[i].region_off + chunk_off16(pa.s[i], cb);

        const int n_items = tiles_here * n_items_per_tile;
        const int it0 = (warp - item_base % kConsumerWarps + kConsumerWarps) % kConsumerWarps;
        item_base += n_items;
        for (int it = it0; it < n_items; it += kConsumerWarps) {
            const int tile = it / n_items_per_tile;
            const int rem = it - tile * n_items_per_tile;
            const int oct = rem / P;
            const int part = rem - oct * P;
            const int q0 = (P == 1) ? 0 : pa.q_bounds[part];
            const int q1 = (P == 1) ? nq : pa.q_bounds[part + 1];
            MmaRow<FMT> ra, rb;
            ra.init(ub[0], NS > 1 ? ub[NS - 1] : 0u, nq, pa.row_bytes, tile * 4 + (row_a >> 2), row_a & 3, tq, q0);
            rb.init(ub[0], NS > 1 ? ub[NS - 1] : 0u, nq, pa.row_bytes, tile * 4 + (row_b >> 2), row_b & 3, tq, q0);
            // this lane's B token (g) and C tokens (2 tq, 2 tq + 1) of the octet
            const int tb = oct * 8 + g;
            const int tc0 = oct * 8 + 2 * tq, tc1 = tc0 + 1;
            const bool vb = tb < ntok;
            // bytes 8 tq .. 8 tq + 7 of each slice's permuted codes: plane A (tq 0, 1) or B (tq 2, 3)
            const uint32_t xb = xbase + static_cast<uint32_t>(vb ? tb : 0) * xa_stride +
                                (tq >= 2 ? static_cast<uint32_t>(K >> 1) : 0u) + static_cast<uint32_t>(q0) * 16u +
                                static_cast<uint32_t>(tq & 1) * 8u;
            const uint32_t xc0 = xbase + static_cast<uint32_t>(tc0 < ntok ? tc0 : 0) * xa_stride + xs_off;
            const uint32_t xc1 = xbase + static_cast<uint32_t>(tc1 < ntok ? tc1 : 0) * xa_stride + xs_off;
            // operands of one group, loaded one group ahead of the MMA that uses them (the
            // shared loads are volatile, so the overlap has to be written out)
            struct In {
                uint32_t wa, wb, ma, mb;
                uint2 b;
                float xs0, xs1, e0, e1;
            };
            auto load = [&](int q, In& d) {
                const uint32_t dq = static_cast<uint32_t>(q - q0);
                d.wa = ra.word_at(q, dq);
                d.wb = rb.word_at(q, dq);
                d.b = vb ? lds64(xb + dq * 16u) : make_uint2(0u, 0u);
                const uint32_t qo = 4u * static_cast<uint32_t>(q);
                d.xs0 = ldsf(xc0 + qo);
                d.xs1 = ldsf(xc1 + qo);
                if constexpr (FMT == kFmtQ4K) {
                    d.e0 = small_int_to_float(static_cast<int>(lds32(xc0 + 2u * nq4 + qo)));
                    d.e1 = small_int_to_float(static_cast<int>(lds32(xc1 + 2u * nq4 + qo)));
                } else {
                    d.ma = ra.meta_at(dq);
                    d.mb = rb.meta_at(dq);
                    d.e0 = ldsf(xc0 + nq4 + qo);
                    d.e1 = ldsf(xc1 + nq4 + qo);
                }
            };
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            In cur, nxt;
            if (q0 < q1) load(q0, cur);
            for (int q = q0; q < q1; ++q) {
                if (q + 1 < q1) load(q + 1, nxt);
                uint32_t a0, a2, a1, a3;
                expand_nibbles(cur.wa, a0, a2);
                expand_nibbles(cur.wb, a1, a3);
                int c[4] = {0, 0, 0, 0};
                mma_s8_m16n8k32(c, a0, a1, a2, a3, cur.b.x, cur.b.y);
                if constexpr (FMT == kFmtQ4K) {
                    // part = (d*sc)*dot - (dmin*m)*xsum; y += part * xs  (gemv_q4_avx2.cpp:294-329)
                    const float2 fa = ra.factors(q), fb = rb.factors(q);
                    acc[0] = __fmaf_rn(__fsub_rn(__fmul_rn(fa.x, small_int_to_float(c[0])), __fmul_rn(fa.y, cur.e0)), cur.xs0, acc[0]);
                    acc[1] = __fmaf_rn(__fsub_rn(__fmul_rn(fa.x, small_int_to_float(c[1])), __fmul_rn(fa.y, cur.e1)), cur.xs1, acc[1]);
                    acc[2] = __fmaf_rn(__fsub_rn(__fmul_rn(fb.x, small_int_to_float(c[2])), __fmul_rn(fb.y, cur.e0)), cur.xs0, acc[2]);
                    acc[3] = __fmaf_rn(__fsub_rn(__fmul_rn(fb.x, small_int_to_float(c[3])), __fmul_rn(fb.y, cur.e1)), cur.xs1, acc[3]);
                } else {
                    // dot*(ws*xs) - (wz*ws)*xss, as the single-token kernel combines a group
                    const float2 sa = half2_bits_to_float2(cur.ma), sb = half2_bits_to_float2(cur.mb);  // (scale, zero)
                    const float za = __fmul_rn(sa.y, sa.x), zb = __fmul_rn(sb.y, sb.x);
                    acc[0] = __fmaf_rn(small_int_to_float(c[0]), __fmul_rn(sa.x, cur.xs0), acc[0]);
                    acc[0] = __fmaf_rn(-za, cur.e0, acc[0]);
                    acc[1] = __fmaf_rn(small_int_to_float(c[1]), __fmul_rn(sa.x, cur.xs1), acc[1]);
                    acc[1] = __fmaf_rn(-za, cur.e1, acc[1]);
                    acc[2] = __fmaf_rn(small_int_to_float(c[2]), __fmul_rn(sb.x, cur.xs0), acc[2]);
                    acc[2] = __fmaf_rn(-zb, cur.e0, acc[2]);
                    acc[3] = __fmaf_rn(small_int_to_float(c[3]), __fmul_rn(sb.x, cur.xs1), acc[3]);
                    acc[3] = __fmaf_rn(-zb, cur.e1, acc[3]);
                }
                cur = nxt;
            }
            const long long row0 = (cb + tile * 4) * 4;  // first row of the tile
            bool finish = true;
            if (P > 1) {
                const int slot = (s * TPC + tile) * kOct + oct;
                float* sp = s_part + (static_cast<size_t>(slot) * P + part) * 128;
                sp[row_a * 8 + 2 * tq] = acc[0];
                sp[row_a * 8 + 2 * tq + 1] = acc[1];
                sp[row_b * 8 + 2 * tq] = acc[2];
                sp[row_b * 8 + 2 * tq + 1] = acc[3];
                __syncwarp();
                int prev = 0;
                if (lane == 0) {
                    __threadfence_block();
                    prev = atomicAdd(&s_cnt[slot], 1);
                }
                prev = __shfl_sync(0xffffffffu, prev, 0);
                finish = (prev == P - 1);
                if (finish) {
                    __threadfence_block();
                    const float* base = s_part + static_cast<size_t>(slot) * P * 128;
                    float v[4] = {0.f, 0.f, 0.f, 0.f};
                    for (int p2 = 0; p2 < P; ++p2) {
                        const float* pp = base + p2 * 128;
                        v[0] += pp[row_a * 8 + 2 * tq];
                        v[1] += pp[row_a * 8 + 2 * tq + 1];
                        v[2] += pp[row_b * 8 + 2 * tq];
                        v[3] += pp[row_b * 8 + 2 * tq + 1];
                    }
#pragma unroll
                    for (int i = 0; i < 4; ++i) acc[i] = v[i];
                    __syncwarp();
                    if (lane == 0) s_cnt[slot] = 0;  // re-arm for the stage's next use
                }
            }
            if (finish) {
                const long long ra_row = row0 + row_a, rb_row = row0 + row_b;
                if (tc0 < ntok) {
                    if (ra_row < M) ga.y[static_cast<long long>(tc0) * M + ra_row] = acc[0];
                    if (rb_row < M) ga.y[static_cast<long long>(tc0) * M + rb_row] = acc[2];
                }
                if (tc1 < ntok) {
                    if (ra_row < M) ga.y[static_cast<long long>(tc1) * M + ra_row] = acc[1];
                    if (rb_row < M) ga.y[static_cast<long long>(tc1) * M + rb_row] = acc[3];
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == S) {
            s = 0;
            ++use;
        }
    }
}

// ---------------------------------------------------------------------------
// host: plan and launch (one CTA per SM, tile-aligned chunks of about the target size)
// ---------------------------------------------------------------------------
// whether two 16-row stages, the token A8 areas and the K-split partials fit the shared-memory
// budget (long rows, e.g. K = 8192 with 10 tokens, do not: the caller then uses the lane-dot path)
inline bool mma_plan_fits(const StreamIn* in, int n_streams, int K, int gs, int n_tokens) {
    uint32_t stage = 0;
    for (int i = 0; i < n_streams; ++i) stage += round_up(static_cast<uint32_t>(4 * in[i].unit_bytes + 48), 16);
    const uint32_t xa = xarea_layout_bytes(K, gs, false) * static_cast<uint32_t>(n_tokens);
    const uint32_t split = round_up(2u * 2u * (8u * 512u + 4u), 128);
    return static_cast<long long>(round_up(kBarBytes + xa, 128)) + 2LL * stage + split <= kSmemBudget;
}

template <int FMT, int PRO, int NT>
int launch_stream_gemv_mma(const StreamIn* in, int n_streams, long long n_units, GemvArgs ga, cudaStream_t stream,
                           const LaunchOpts& opt = LaunchOpts()) {
    if (ga.n_tokens < 1 || ga.n_tokens > NT) return set_error(kEinval, "internal: token count out of range");
    if (n_units <= 0) return kOk;
    if (n_units > 0x7fffffffLL) return set_error(kEinval, "too many rows");
    if (n_streams != FmtTraits<FMT>::kStreams) return set_error(kEinval, "internal: stream count mismatch");
    PipeArgs pa;
    std::memset(&pa, 0, sizeof(pa));
    pa.n_units = static_cast<int>(n_units);
    long long ub_sum = 0;
    for (int i = 0; i < n_streams; ++i) {
        if (!aligned16(in[i].base)) return set_error(kEinval, "weight buffers must be 16-byte aligned device pointers");
        ub_sum += in[i].unit_bytes;
    }
    const long long tiles = (n_units + 3) / 4;
    int grid = sm_count();
    if (grid > tiles) grid = static_cast<int>(tiles);
    const long long tiles_per_cta = (tiles + grid - 1) / grid;
    long long tpc = opt.chunk_target / (4 * (ub_sum > 0 ? ub_sum : 1));  // tiles per chunk
    if (tpc < 1) tpc = 1;
    if (tpc > tiles_per_cta) tpc = tiles_per_cta;
    const int nq = ga.K / 32;
    const int n_oct = (ga.n_tokens + 7) / 8;
    // K parts: enough work items per chunk for every consumer warp
    int parts = 1;
    while (parts < 8 && parts * 2 <= nq && tpc * n_oct * parts < kConsumerWarps) parts *= 2;
    const uint32_t xa = xarea_layout_bytes(ga.K, ga.gs, false) * static_cast<uint32_t>(ga.n_tokens);
    uint32_t stage_bytes = 0, split_bytes = 0;
    int stages = 0;
    for (;;) {
        stage_bytes = 0;
        for (int i = 0; i < n_streams; ++i) {
            pa.s[i].region_off = stage_bytes;
            stage_bytes += round_up(static_cast<uint32_t>(4 * tpc * in[i].unit_bytes + 48), 16);
        }
        const long long avail = static_cast<long long>(kSmemBudget) - kBarBytes - xa;
        const uint32_t split_per_stage =
            static_cast<uint32_t>(tpc * (NT / 8) * (parts > 1 ? parts * 128 * 4 + 4 : 0));
        stages = avail > 0 ? static_cast<int>(avail / (stage_bytes + split_per_stage)) : 0;
        if (stages > kMaxStages) stages = kMaxStages;
        split_bytes = round_up(static_cast<uint32_t>(stages) * split_per_stage, 128);
        if (stages >= 2 || tpc == 1) break;
        tpc = tpc / 2 > 0 ? tpc / 2 : 1;
    }
    if (stages < 2) return set_error(kEinval, "in_features too large for the shared-memory pipeline");
    for (int i = 0; i < n_streams; ++i) {
        pa.s[i].base = static_cast<const uint8_t*>(in[i].base);
        pa.s[i].unit_bytes = in[i].unit_bytes;
        pa.s[i].total_bytes = in[i].total_bytes;
    }
    pa.units_per_chunk = static_cast<int>(4 * tpc);
    pa.n_stages = stages;
    pa.k_parts = parts;
    for (int p = 0; p <= parts; ++p) pa.q_bounds[p] = static_cast<int>(static_cast<long long>(nq) * p / parts);
    pa.inv_ipu = 1.0f;
    pa.seg_bytes = stage_bytes;
    pa.stage_bytes = stage_bytes;
    pa.xarea_off = kBarBytes;
    pa.stage_off = round_up(kBarBytes + xa, 128);
    pa.split_off = pa.stage_off + static_cast<uint32_t>(stages) * stage_bytes;
    pa.row_bytes = opt.row_bytes;
    if (!aligned16(ga.x)) return set_error(kEinval, "activations must be 16-byte aligned");
    const uint32_t smem = pa.split_off + split_bytes;
    if (smem > kSmemBudget) return set_error(kEinval, "internal: tensor-core GEMV plan exceeds shared memory");
    ga.status = device_status_ptr();
    if (!ga.status) return set_error(kEcuda, "cannot resolve the device status word");
    auto kern = k_stream_gemv_mma<FMT, PRO, NT>;
    {
        static std::mutex mu;
        static bool configured[64] = {false};
        int dev = 0;
        cudaGetDevice(&dev);
        std::lock_guard<std::mutex> lk(mu);
        if (dev >= 0 && dev < 64 && !configured[dev]) {
            ASDSL_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget + 1024));
            configured[dev] = true;
        }
    }
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (opt.pdl || launch_policy().pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    ASDSL_CUDA(cudaLaunchKernelEx(&cfg, kern, pa, ga));
    return kOk;
}

}  // namespace asdsl
