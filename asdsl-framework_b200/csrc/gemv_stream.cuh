// gemv_stream.cuh -- the W4A8 / W4A32 decode GEMV family on sm_100a.
//
// One kernel template serves every weight format of the reference's decode
// path.  A weight matrix is a set of byte "streams" (preq2: quant + meta;
// banded Q4_128: quant + scales; packed: nibbles + scales + biases; the
// row-major block formats: one stream), each made of fixed-size "units"
// (a band of 4 rows, or one row for the fp32-activation packed format).
// Each CTA owns a contiguous run of units, so each of its streams is ONE
// contiguous span of HBM.  A single producer thread walks that span in large
// 1-D bulk copies (cp.async.bulk, no multicast; tens of KB per copy, which is
// what streams HBM at full rate) into a ring of shared-memory stages guarded
// by mbarriers, and every consumer warp takes work items from every stage.
//
// Work item = (band of 4 rows, K slice, segment).  Lane l walks 32-weight
// slices q = l, l+32, ... of all four rows at once, two slices in flight, so
// a slice's int8 activation record is loaded once for four rows; rows are
// visited in a lane-rotated order that keeps 128-bit shared loads bank-
// conflict free; nibbles are masked in place (LOP3) and dotted with dp4a; a
// 6-shuffle reduce-scatter leaves row j of the band in lane 8*j.  When a unit
// is split in several items (K slices, or the gate and up halves of the fused
// SiLU), the last item to finish sums the partials in a fixed order.
//
// The activation prologue is fused: each CTA quantizes the input vector to
// int8 with the reference's A8 rounding (optionally after RMSNorm) while its
// first weight stages stream in.  Programmatic dependent launch: the producer
// starts streaming weights before griddepcontrol.wait, consumers wait before
// touching any activation or output, so a kernel can overlap its predecessor.
//
// Reference formats and math (asdsl/kernels/native/):
//   preq2  gemv_preq2_avx2.cpp:196-297    preq   gemv_q4_preq_restored.cpp:305-473
//   Q4_128 gemv_q4_128.cpp:94-257          S256   gemv_q4_s256.cpp:83-209
//   Q4_K   gemv_q4_avx2.cpp:283-420        packed gemv_q4_avx2.cpp:665-749
#pragma once

#include "common.cuh"
#include "exact_math.cuh"

namespace asdsl {

enum WeightFormat : int {
    kFmtPreq2 = 0,    // meta [M][ng][4] + quant [ceil(M/4)][ng][64], gs 32
    kFmtPreq = 1,     // [M][ng][20] blocks, gs 32
    kFmtQ4_128 = 2,   // [M][K/128][66] blocks, symmetric, implicit zero 8 (reference bytes)
    kFmtS256 = 3,     // [M][K/256][144] blocks, 8 fp16 sub-scales, zero 8, A8 gs 32
    kFmtQ4K = 4,      // [M][K/256][144] reference-interpretation Q4_K, own A8
    kFmtPacked = 5,   // nibbles [M][K/2] + fp32 scales [M][ng] + fp32 biases [M][ng], fp32 x
    kFmtQ128B = 6,    // banded Q4_128: quant [nb][K/128][4][64] + scales [nb][K/128][4] fp16
    kFmtPreq2X = 7,   // preq2 bytes, every row summed in the reference's compiled order (exact mode);
    kFmtPreq2X2 = 8,  // 7..10: a unit of 1, 2, 4, 8 bands, each thread owning 1, 2, 4, 8 of a row's
    kFmtPreq2X4 = 9,  // eight int32 dot lanes (exact_lpt)
    kFmtPreq2X8 = 10,
};

__host__ __device__ constexpr bool is_exact_fmt(int fmt) { return fmt >= kFmtPreq2X && fmt <= kFmtPreq2X8; }
__host__ __device__ constexpr int exact_lpt(int fmt) { return 1 << (fmt - kFmtPreq2X); }

enum Prologue : int {
    kProA8 = 0,     // fp32 x -> A8 (gs 32 or 128)
    kProQ8 = 1,     // caller-quantized x (int8 + per-group fp32 scale)
    kProRmsA8 = 2,  // RMSNorm(x) * w then A8
    kProQ4K = 3,    // the Q4_K kernel's own A8 (half-away, clamp +-127)
    kProF32 = 4,    // fp32 x kept as is, plus per-group sums (packed W4A32)
    kProA8X = 5,    // kProA8 for kFmtPreq2X*: codes in lane order (4 per 32-bit word, see rows_exact)
    kProRmsA8X = 6, // kProRmsA8 for kFmtPreq2X: the reference's compiled RMSNorm, then A8 in lane order
};

enum Epilogue : int {
    kEpiStore = 0,   // y[row] = v
    kEpiResid = 1,   // resid[row] += v (in place; the decode residual stream)
    kEpiSilu = 2,    // paired gate/up: h[i] = silu(gate_i) * up_i
    kEpiArgmax = 3,  // y[row] = v (optional) + global first-max argmax
    kEpiSiluX = 4,   // kEpiSilu with swiglu_inplace's compiled arithmetic (exact mode)
};

__host__ __device__ constexpr bool pro_is_rms(int pro) { return pro == kProRmsA8 || pro == kProRmsA8X; }
__host__ __device__ constexpr bool pro_is_lane_order(int pro) { return pro == kProA8X || pro == kProRmsA8X; }
__host__ __device__ constexpr bool epi_is_silu(int epi) { return epi == kEpiSilu || epi == kEpiSiluX; }

// measured on B200 (decode chains and lm_head): one 17-warp CTA per SM with
// 64 KB stages beats two 9-warp CTAs
#ifndef ASDSL_CONSUMER_WARPS
#define ASDSL_CONSUMER_WARPS 16
#endif
#ifndef ASDSL_CTAS_PER_SM
#define ASDSL_CTAS_PER_SM 1
#endif
constexpr int kConsumerWarps = ASDSL_CONSUMER_WARPS;
constexpr int kCtasPerSm = ASDSL_CTAS_PER_SM;
#ifndef ASDSL_MT_GROUP
// multi-token GEMVs: activation rows per weight-slice load (each group keeps 4 x rows accumulators)
#define ASDSL_MT_GROUP 4
#endif
constexpr int kThreads = 32 * (kConsumerWarps + 1);  // + one producer warp
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kConsumerThreads = 32 * kConsumerWarps;
constexpr int kMaxStages = 24;
constexpr int kMaxStreams = 3;

template <int FMT>
struct FmtTraits {
    static constexpr int kStreams =
        (FMT == kFmtPreq2 || is_exact_fmt(FMT) || FMT == kFmtQ128B) ? 2 : (FMT == kFmtPacked ? 3 : 1);
    static constexpr int kRowsPerUnit = (FMT == kFmtPacked) ? 1 : (is_exact_fmt(FMT) ? 4 * exact_lpt(FMT) : 4);
};

struct StreamDesc {
    const uint8_t* base;   // 16-byte aligned
    long long unit_bytes;  // bytes per unit
    long long total_bytes; // stream length (clamps the last unit)
    uint32_t region_off;   // offset of this stream's region inside a segment of a stage
    uint32_t pad;
};

struct PipeArgs {
    StreamDesc s[kMaxStreams];
    int n_units;          // units per segment
    int pair_unit_off;    // paired (gate/up) mode: segment 1 starts this many units later
    int units_per_chunk;
    int n_stages;
    int k_parts;          // work items per unit and segment: the K range in k_parts slices
    int q_bounds[9];      // slice boundaries (in 32-weight slices) of the k_parts parts
    float inv_ipu;        // 1 / (k_parts * segments), for division-free item indexing
    uint32_t seg_bytes;   // bytes of one segment inside a stage
    uint32_t stage_bytes; // bytes of one stage (1 or 2 segments)
    uint32_t xarea_off;   // dynamic smem offsets
    uint32_t stage_off;
    uint32_t split_off;   // K-split / segment-split partials
    int row_bytes;        // row-major block formats: bytes of one row
};

struct GemvArgs {
    const float* x;        // fp32 activation
    const int8_t* xq;      // kProQ8: int8 activation
    const float* xs_in;    // kProQ8: per-group scales
    const float* norm_w;   // kProRmsA8
    float eps;
    int K;                 // in_features
    int M;                 // out rows (per segment)
    int gs;                // activation group size (32, or 128 for the Q4_128 formats)
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
    int n_tokens;          // multi-token kernels (NT > 1): activation rows x[t][K] -> y[t][M]
    // argmax exchange with the peer GPUs of a row-sharded lm_head (null = single GPU):
    // slot buffers [2 parities][world] of packed (max bits | index << 32 | epoch << 56)
    unsigned long long* const* xchg_peers;  // [world] every rank's slot buffer (peer mappings)
    unsigned long long* xchg_self;          // this rank's slot buffer
    int* xchg_epoch;                        // device-resident step counter of the exchange
    int xchg_world, xchg_rank;
    // optional %globaltimer stamps of the exchange, [slot = step & mask][4]: consumers released,
    // local argmax done, own word stored to every peer, every peer's word seen (null = off)
    unsigned long long* xchg_stamps;
    int xchg_stamp_mask;
    // multi-token kernels: the tokens' A8 areas, quantized once by k_quant_tokens in the layout
    // of the shared-memory areas (n_tokens x xarea_layout_bytes); null = each CTA quantizes
    const uint8_t* xa_pre;
    // reference-exact mode (kProRmsA8X, kEpiSiluX): the host CPU's RSQRTSS / RCPPS tables
    ExactTabs ex;
    int exact_inter;  // kFmtPreq2X*: the weights are in the exact (group-interleaved) layout
    unsigned int tl_id;  // host-side launch number, carried into the timeline records
};

// ---------------------------------------------------------------------------
// Optional per-CTA timeline of the streaming GEMVs (asdsl_b200_timeline_set): while a buffer is
// set, every CTA takes the next slot of its block (one atomic on a per-block counter, so CTAs do
// not contend) and one thread per event writes {%globaltimer, event | kernel template << 4,
// launch number} into record [block][slot][event].  The counterpart of the reference's
// ASDSL_ENGINE_PROFILE breakdown for the per-op chain; off (null buffer) by default.
// ---------------------------------------------------------------------------
#ifndef ASDSL_B200_TIMELINE
#define ASDSL_B200_TIMELINE 0  // the timeline build (libasdsl_b200_timeline.so) defines it as 1
#endif
// the records exist only in the timeline build: with them compiled in but switched off, the hot
// kernels still lost ~3 % (config-1 layer step, B200) to the extra registers and branches
constexpr bool kTimeline = ASDSL_B200_TIMELINE != 0;

struct TlRec {
    unsigned long long t;
    uint32_t code, id;
};
constexpr int kTlEvents = 16;     // record slots per CTA (events 0..9 used)
constexpr int kTlMaxBlocks = 1024;
// constant memory: every CTA reads these at its start, before its first barrier; the per-SM
// constant cache keeps that read off the memory system once a kernel has run (a global variable
// cost every CTA an L2 round trip before its producer could start streaming)
__constant__ TlRec* g_tl_buf;     // [kTlMaxBlocks][slots][kTlEvents], null = off
__constant__ uint32_t* g_tl_cnt;  // [kTlMaxBlocks] slots taken per block
__constant__ uint32_t g_tl_slots;
enum TlEvent : uint32_t {
    kTlReduced = 0,   // RMSNorm prologues: the sum of squares reduced (thread 0)
    kTlStart = 1,     // CTA initialized (barriers set up)
    kTlWaited = 2,    // consumers past the dependency wait (previous kernel complete)
    kTlPrologue = 3,  // activation prologue done
    kTlConsumed = 4,  // consumer warp 0 through its last work item
    kTlEnd = 5,       // every consumer warp done
    kTlProduced = 6,  // producer issued its last copy
    kTlXLoaded = 7,   // thread 0's first activation values arrived (prologue)
    kTlFirstFull = 8, // consumer thread 0 past the full barrier of the CTA's first chunk
    kTlLastFull = 9,  // ... and of its last chunk (all of the CTA's weights landed)
    kTlXAll = 10,     // the latest consumer warp's first activation values arrived (prologue)
    // k_attention_exact (template code 15): RoPE + KV quantization, scores, maxima, weights, tile sums
    kTlAttnRope = 11,
    kTlAttnScores = 12,
    kTlAttnMaxima = 13,
    kTlAttnWeights = 14,
    kTlAttnSums = 15,
};

// a CTA's timeline slot with its record code and launch number (slot ~0u: off)
struct TlCtx {
    uint32_t slot, code, id;
};

// the CTA's slot (thread 0, before the CTA's first barrier), or ~0u when off / full
__device__ __forceinline__ uint32_t tl_slot() {
    if (!kTimeline || g_tl_buf == nullptr || blockIdx.x >= static_cast<unsigned>(kTlMaxBlocks)) return ~0u;
    const uint32_t k = atomicAdd(g_tl_cnt + blockIdx.x, 1u);
    return k < g_tl_slots ? k : ~0u;
}

__device__ __forceinline__ void tl_put(const TlCtx& c, uint32_t ev, unsigned long long t = 0) {
    if (!kTimeline || c.slot == ~0u) return;
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    TlRec r;
    r.t = t ? t : globaltimer_ns();
    r.code = ev | c.code | (smid << 24);
    r.id = c.id;
    g_tl_buf[(static_cast<size_t>(blockIdx.x) * g_tl_slots + c.slot) * kTlEvents + ev] = r;
}

template <int FMT, int PRO, int EPI, int NT>
__device__ __forceinline__ void tl_rec(uint32_t slot, uint32_t ev, uint32_t id) {
    constexpr uint32_t code = (static_cast<uint32_t>(FMT) << 4) | (static_cast<uint32_t>(PRO) << 8) |
                              (static_cast<uint32_t>(EPI) << 12) | (static_cast<uint32_t>(NT) << 16);
    tl_put(TlCtx{slot, code, id}, ev);
}

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

// start - a0 of chunk_span for a chunk starting at unit u inside the stream (its start never
// clamps there): the low four bits of u * unit_bytes, which 32-bit arithmetic gives exactly
__device__ __forceinline__ uint32_t chunk_off16(const StreamDesc& sd, long long u) {
    return (static_cast<uint32_t>(u) * static_cast<uint32_t>(sd.unit_bytes)) & 15u;
}

// ---------------------------------------------------------------------------
// shared-memory activation area
//   x8[K]      int8 codes, permuted per 32-slice, in two planes of K/2 bytes: plane A holds bytes
//              0-15 of every slice's 32 permuted codes, plane B bytes 16-31, so the 16-byte loads of
//              32 lanes on 32 consecutive slices hit every bank once (no 2-way conflict)
//   xs[K/32]   A8 scale of each 32-slice's group (replicated for gs 128)
//   xss[K/32]  (float)sum(codes of the slice) * xs
//   xsi[K/32]  sum(codes of the slice)
//   red[32]    reduction scratch
//   kProF32:   xf[K] fp32 x and sx[K/gs] per-group sums instead of the codes
// ---------------------------------------------------------------------------
struct XArea {
    float* xf;
    int8_t* x8;
    float* xs;
    float* xss;
    int* xsi;
    float* sx;
    float* red;
};

// the same area as 32-bit shared-window addresses (for explicit ld.shared)
struct XAddr {
    uint32_t x8, x8b, xs, xss, xsi;  // x8b: plane B of the codes (x8 + K/2)
};

__host__ __device__ __forceinline__ uint32_t xarea_layout_bytes(int K, int gs, bool f32) {
    const uint32_t nq = static_cast<uint32_t>(K / 32);
    const uint32_t ng = static_cast<uint32_t>(K / gs);
    uint32_t b = f32 ? 4u * K + 4u * ng : ((static_cast<uint32_t>(K) + 15u) & ~15u) + 12u * nq;
    b = (b + 15u) & ~15u;
    b += 4u * 32u;  // red
    return (b + 127u) & ~127u;
}

__device__ __forceinline__ XArea xarea_layout(uint8_t* base, int K, int gs, bool f32) {
    XArea a;
    const int nq = K / 32;
    const int ng = K / gs;
    uint8_t* p = base;
    if (f32) {
        a.xf = reinterpret_cast<float*>(p);
        a.sx = a.xf + K;
        p = reinterpret_cast<uint8_t*>(a.sx + ng);
        a.x8 = nullptr;
        a.xs = a.xss = nullptr;
        a.xsi = nullptr;
    } else {
        a.xf = nullptr;
        a.sx = nullptr;
        a.x8 = reinterpret_cast<int8_t*>(p);
        p += (K + 15) & ~15;
        a.xs = reinterpret_cast<float*>(p);
        a.xss = a.xs + nq;
        a.xsi = reinterpret_cast<int*>(a.xss + nq);
        p = reinterpret_cast<uint8_t*>(a.xsi + nq);
    }
    uintptr_t r = reinterpret_cast<uintptr_t>(p);
    r = (r + 15) & ~uintptr_t(15);
    a.red = reinterpret_cast<float*>(r);
    return a;
}

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerThreads) : "memory");
}

// ---------------------------------------------------------------------------
// fused activation prologue (consumer warps), straight from global memory.
// Quad-parallel: each thread owns 4 consecutive elements; an A8 group of gs
// elements is gs/4 consecutive threads of one warp.
// ---------------------------------------------------------------------------
// activation load: read-only path in a standalone GEMV; L2 (coherent across SMs) when the
// activation is produced by other CTAs of the same persistent kernel
template <bool kCoherent>
__device__ __forceinline__ float4 load_x4(const float4* p) {
    if constexpr (kCoherent) return __ldcg(p);
    else return __ldg(p);
}
template <bool kCoherent>
__device__ __forceinline__ float load_x1(const float* p) {
    if constexpr (kCoherent) return __ldcg(p);
    else return __ldg(p);
}

// quads of the activation per consumer thread held in registers by the prologue (up to K = 8192)
constexpr int kRegIters = 4;

template <int PRO, bool kCoherent = false>
__device__ void run_prologue(const GemvArgs& ga, XArea xa, int ctid, TlCtx tl = TlCtx{~0u, 0u, 0u}) {
    const int K = ga.K;
    const int lane = ctid & 31;

    if constexpr (PRO == kProF32) {
        for (int i = ctid * 4; i < K; i += kConsumerThreads * 4)
            *reinterpret_cast<float4*>(xa.xf + i) = __ldg(reinterpret_cast<const float4*>(ga.x + i));
        consumer_sync();
        // per-group sums in the reference's 8-lane order (gemv_q4_avx2.cpp:677-685)
        const int gs = ga.gs;
        const int ng = K / gs;
        for (int g = ctid; g < ng; g += kConsumerThreads) {
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
        const int nquads = K >> 2;
        const int gs = ga.gs;     // 32 or 128
        const int tpg = gs >> 2;  // threads per A8 group: 8 or 32
        // up to K = 8192 every thread's quads are loaded once, into registers: the RMSNorm sum of
        // squares and the quantization then share one round trip to memory
        const bool in_regs = (PRO != kProQ8) && nquads <= kRegIters * kConsumerThreads;
        float4 xr[kRegIters];
        if (in_regs) {
#pragma unroll
            for (int k = 0; k < kRegIters; ++k) {
                const int t = k * kConsumerThreads + ctid;
                xr[k] = (t < nquads) ? load_x4<kCoherent>(reinterpret_cast<const float4*>(ga.x) + t)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            if (tl.slot != ~0u) {
                // the records wait for the loads: thread 0's arrival, and the latest warp's
                __shared__ unsigned long long s_xall;
                if (ctid == 0) s_xall = 0ull;
                consumer_sync();
                asm volatile("" ::"f"(xr[0].x), "f"(xr[1].x), "f"(xr[2].x), "f"(xr[3].x));
                const unsigned long long tx = globaltimer_ns();
                if (ctid == 0) tl_put(tl, kTlXLoaded, tx);
                if ((ctid & 31) == 0) atomicMax(&s_xall, tx);
                consumer_sync();
                if (ctid == 0) tl_put(tl, kTlXAll, s_xall);
            }
        }
        float inv_rms = 1.0f;
        if constexpr (PRO == kProRmsA8X) {
            // rmsnorm_f32 as compiled (unified_engine.cpp:499-524): lane l of one 8-wide vector
            // accumulates x[8i+l]^2 by FMA in order of i; hsum256_ps fold; sum/n + eps; RSQRTSS +
            // Newton.  The CTA stages x in shared memory (behind the A8 area, one coalesced pass),
            // then eight threads run the eight sequential lane chains from there.
            float* xst = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xa.x8) + xarea_layout_bytes(K, ga.gs, false));
            if (in_regs) {
#pragma unroll
                for (int k = 0; k < kRegIters; ++k) {
                    const int t = k * kConsumerThreads + ctid;
                    if (t < nquads) reinterpret_cast<float4*>(xst)[t] = xr[k];
                }
            } else {
                for (int t = ctid; t < nquads; t += kConsumerThreads)
                    reinterpret_cast<float4*>(xst)[t] = load_x4<kCoherent>(reinterpret_cast<const float4*>(ga.x) + t);
            }
            consumer_sync();
            if (ctid < 8) {
                float acc = 0.0f;
                const float* xp = xst + ctid;
#pragma unroll 16
                for (int i = 0; i < (K >> 3); ++i) {
                    const float v = xp[8 * i];
                    acc = __fmaf_rn(v, v, acc);
                }
                const float a = __fadd_rn(acc, __shfl_xor_sync(0xffu, acc, 4));  // v_l + v_{l+4}
                const float b = __fadd_rn(a, __shfl_xor_sync(0xffu, a, 1));      // (a0+a1), (a2+a3)
                const float h = __fadd_rn(b, __shfl_xor_sync(0xffu, b, 2));      // (a0+a1) + (a2+a3)
                if (ctid == 0)
                    xa.red[0] = exact_nr_rsqrt(__fadd_rn(__fdiv_rn(h, static_cast<float>(K)), ga.eps), ga.ex.rsqrt);
            }
            consumer_sync();
            inv_rms = xa.red[0];
            if (ctid == 0) tl_put(tl, kTlReduced);
        } else if constexpr (PRO == kProRmsA8) {
            // inv = 1/sqrt(sum(x^2)/n + eps)  (unified_engine.cpp:499-513)
            float ss = 0.0f;
            auto acc = [&](const float4& f) {
                ss = __fmaf_rn(f.x, f.x, ss);
                ss = __fmaf_rn(f.y, f.y, ss);
                ss = __fmaf_rn(f.z, f.z, ss);
                ss = __fmaf_rn(f.w, f.w, ss);
            };
            if (in_regs) {
#pragma unroll
                for (int k = 0; k < kRegIters; ++k) acc(xr[k]);
            } else {
                for (int t = ctid; t < nquads; t += kConsumerThreads)
                    acc(load_x4<kCoherent>(reinterpret_cast<const float4*>(ga.x) + t));
            }
            ss = warp_sum(ss);
            if (lane == 0) xa.red[ctid >> 5] = ss;
            consumer_sync();
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) tot = __fadd_rn(tot, xa.red[w]);
            inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(K)), ga.eps)));
            if (ctid == 0) tl_put(tl, kTlReduced);
        }
        // one quad (4 consecutive elements) of thread t: A8 codes into the permuted x8 area and,
        // from the lane holding a 32-slice's first quad, its scale and code sums
        auto quad = [&](int t, const float4* preloaded) {
            const bool live = t < nquads;
            const int e0 = t * 4;
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            int c[4] = {0, 0, 0, 0};
            float scale = 1.0f;
            if constexpr (PRO == kProQ8) {
                if (live) {
                    const char4 q4 = *reinterpret_cast<const char4*>(ga.xq + e0);
                    c[0] = q4.x;
                    c[1] = q4.y;
                    c[2] = q4.z;
                    c[3] = q4.w;
                    scale = __ldg(ga.xs_in + e0 / gs);
                }
            } else {
                if (live) {
                    const float4 f = preloaded ? *preloaded
                                               : load_x4<kCoherent>(reinterpret_cast<const float4*>(ga.x) + t);
                    v[0] = f.x;
                    v[1] = f.y;
                    v[2] = f.z;
                    v[3] = f.w;
                    if constexpr (PRO == kProRmsA8X) {
                        // compiled order: (x * w) * inv
                        const float4 w = __ldg(reinterpret_cast<const float4*>(ga.norm_w) + t);
                        v[0] = __fmul_rn(__fmul_rn(v[0], w.x), inv_rms);
                        v[1] = __fmul_rn(__fmul_rn(v[1], w.y), inv_rms);
                        v[2] = __fmul_rn(__fmul_rn(v[2], w.z), inv_rms);
                        v[3] = __fmul_rn(__fmul_rn(v[3], w.w), inv_rms);
                    } else if constexpr (PRO == kProRmsA8) {
                        const float4 w = __ldg(reinterpret_cast<const float4*>(ga.norm_w) + t);
                        v[0] = __fmul_rn(__fmul_rn(v[0], inv_rms), w.x);
                        v[1] = __fmul_rn(__fmul_rn(v[1], inv_rms), w.y);
                        v[2] = __fmul_rn(__fmul_rn(v[2], inv_rms), w.z);
                        v[3] = __fmul_rn(__fmul_rn(v[3], inv_rms), w.w);
                    }
                }
                float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
                for (int o = 1; o < tpg; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                if constexpr (PRO == kProQ4K) {
                    // gemv_q4_avx2.cpp:377-400: amax < 1e-12 -> scale 0, codes 0;
                    // q = clamp(round_half_away(x * 127/amax), -127, 127)
                    if (amax < 1e-12f) {
                        scale = 0.0f;
                    } else {
                        const float inv = __fdiv_rn(127.0f, amax);
                        scale = __fmul_rn(amax, inv127f());
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            int q = static_cast<int>(roundf(__fmul_rn(v[j], inv)));
                            c[j] = q > 127 ? 127 : (q < -127 ? -127 : q);
                        }
                    }
                } else {
                    // gemv_q4_preq_restored.cpp:529-547
                    if (amax < 1e-9f) {
                        scale = 1.0f;
                    } else {
                        const float inv = __fdiv_rn(127.0f, amax);
                        scale = __fmul_rn(amax, inv127f());
#pragma unroll
                        for (int j = 0; j < 4; ++j) c[j] = a8_code(v[j], inv);
                    }
                }
            }
            if (live && pro_is_lane_order(PRO)) {
                // lane order: the quad is lane (e0 & 31) / 4 of its 32-group; one word of the codes
                // in the byte order rows_exact's nibble words use, [c0, c2, c1, c3]
                *reinterpret_cast<uint32_t*>(xa.x8 + e0) = (c[0] & 0xFFu) | ((c[2] & 0xFFu) << 8) |
                                                           ((c[1] & 0xFFu) << 16) | ((c[3] & 0xFFu) << 24);
            } else if (live) {
                // quad (4 consecutive elements, first one even) -> even word gets c0, c2 and the odd
                // word c1, c3 at byte (e0 & 7) / 2 of the 8-byte pair of its 8 elements; the pairs of
                // elements 0-15 of a slice go to plane A, those of 16-31 to plane B
                const int w8 = ((e0 & 16) ? (ga.K >> 1) : 0) + (e0 >> 5) * 16 + ((e0 & 15) >> 3) * 8 + ((e0 & 7) >> 1);
                *reinterpret_cast<uint16_t*>(xa.x8 + w8) =
                    static_cast<uint16_t>((c[0] & 0xFF) | ((c[2] & 0xFF) << 8));
                *reinterpret_cast<uint16_t*>(xa.x8 + w8 + 4) =
                    static_cast<uint16_t>((c[1] & 0xFF) | ((c[3] & 0xFF) << 8));
            }
            // per 32-slice sums (8 quads)
            int sm = c[0] + c[1] + c[2] + c[3];
            sm += __shfl_xor_sync(0xffffffffu, sm, 1);
            sm += __shfl_xor_sync(0xffffffffu, sm, 2);
            sm += __shfl_xor_sync(0xffffffffu, sm, 4);
            if (live && (t & 7) == 0) {
                const int q = e0 >> 5;
                if constexpr (pro_is_lane_order(PRO)) {
                    // (scale, xsum_scaled) pairs over the xs and xss areas: one 8-byte load per group
                    reinterpret_cast<float2*>(xa.xs)[q] = make_float2(scale, __fmul_rn(static_cast<float>(sm), scale));
                } else {
                    xa.xs[q] = scale;
                    xa.xsi[q] = sm;
                    xa.xss[q] = __fmul_rn(static_cast<float>(sm), scale);
                }
            }
        };
        if (in_regs) {
#pragma unroll
            for (int k = 0; k < kRegIters; ++k) {
                if (k * kConsumerThreads >= nquads) break;  // uniform across the CTA
                quad(k * kConsumerThreads + ctid, &xr[k]);
            }
        } else {
#pragma unroll 2
            for (int base = 0; base < nquads; base += kConsumerThreads) quad(base + ctid, nullptr);
        }
        consumer_sync();
    }
}

// Multi-token prologue: copy the A8 areas that k_quant_tokens wrote (one per token, the layout of
// the shared-memory areas) into shared memory, or quantize every token here when there are none.
template <int PRO>
__device__ void token_prologue(const GemvArgs& ga, uint8_t* area0, uint32_t xa_stride) {
    if (ga.xa_pre != nullptr) {
        const int n16 = static_cast<int>((xa_stride * static_cast<uint32_t>(ga.n_tokens)) >> 4);
        const uint4* src = reinterpret_cast<const uint4*>(ga.xa_pre);
        uint4* dst = reinterpret_cast<uint4*>(area0);
        for (int i = threadIdx.x; i < n16; i += kConsumerThreads) dst[i] = __ldcg(src + i);
        consumer_sync();
        return;
    }
    for (int t = 0; t < ga.n_tokens; ++t) {
        GemvArgs gt = ga;
        gt.x = ga.x + static_cast<size_t>(t) * ga.K;
        run_prologue<PRO>(gt, xarea_layout(area0 + t * xa_stride, ga.K, ga.gs, false), threadIdx.x);
    }
}

// The tokens' A8 areas for a multi-token GEMV, once instead of in every CTA: block t (of
// kConsumerThreads threads, the prologue's barrier width) quantizes token t into
// out + t * xa_stride exactly as the GEMV's own prologue would in shared memory.
template <int PRO>
__global__ void __launch_bounds__(kConsumerThreads) k_quant_tokens(const GemvArgs ga, uint8_t* out,
                                                                 uint32_t xa_stride) {
    grid_dependency_wait();
    grid_launch_dependents();
    GemvArgs gt = ga;
    gt.x = ga.x + static_cast<size_t>(blockIdx.x) * ga.K;
    run_prologue<PRO>(gt, xarea_layout(out + blockIdx.x * xa_stride, ga.K, ga.gs, false), threadIdx.x);
}

// ---------------------------------------------------------------------------
// band compute: 4 rows x K slices [q0, q1).  Accumulates into a[r] the lane's
// partial (acc - corr) of row (r + rot) & 3.
// ---------------------------------------------------------------------------
struct SliceData {
    uint4 xa, xb;
    float xs, xss;
    int xsi;
    uint4 w[4];
    uint32_t m[4];  // per-row scale (and zero) bits, or the Q4_K block address
};

// the activation half of a slice: A8 codes (permuted), group scale, scale*sum, sum
template <int FMT>
__device__ __forceinline__ void slice_load_x(SliceData& d, const XAddr& xs, int q) {
    const uint32_t uq = static_cast<uint32_t>(q);
    d.xa = lds128(xs.x8 + uq * 16u);
    d.xb = lds128(xs.x8b + uq * 16u);
    d.xs = ldsf(xs.xs + 4u * uq);
    d.xss = ldsf(xs.xss + 4u * uq);
    if constexpr (FMT == kFmtQ4K) d.xsi = static_cast<int>(lds32(xs.xsi + 4u * uq));
}

// the weight half of a slice: 4 rows of 32 nibbles and their scale / zero bits
template <int FMT>
__device__ __forceinline__ void slice_load_w(SliceData& d, uint32_t s0, uint32_t s1, int nq, int rs,
                                             const uint32_t rr[4], int q) {
    const uint32_t uq = static_cast<uint32_t>(q);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const uint32_t row = rr[r];
        if constexpr (FMT == kFmtPreq2) {
            // quant band: [ng][4 rows][16 B]; meta band: [4 rows][ng][4 B]
            d.w[r] = lds128(s0 + uq * 64u + row * 16u);
            d.m[r] = lds32(s1 + row * static_cast<uint32_t>(nq) * 4u + uq * 4u);
        } else if constexpr (FMT == kFmtQ128B) {
            // quant band: [K/128][4 rows][64 B]; scales band: [K/128][4 rows] fp16
            const uint32_t g = uq >> 2, cq = uq & 3u;
            d.w[r] = lds128(s0 + g * 256u + row * 64u + cq * 16u);
            d.m[r] = lds16(s1 + g * 8u + row * 2u);
        } else if constexpr (FMT == kFmtQ4_128) {
            const uint32_t g = uq >> 2, cq = uq & 3u;
            const uint32_t blk = s0 + row * static_cast<uint32_t>(rs) + g * 66u;
            d.w[r] = lds128_a2s(blk + 2u + cq * 16u);
            d.m[r] = lds16(blk);
        } else if constexpr (FMT == kFmtPreq) {
            const uint32_t b = s0 + row * static_cast<uint32_t>(rs) + uq * 20u;
            d.m[r] = lds32(b);
            d.w[r] = make_uint4(lds32(b + 4), lds32(b + 8), lds32(b + 12), lds32(b + 16));
        } else if constexpr (FMT == kFmtS256) {
            const uint32_t k8 = uq & 7u;
            const uint32_t blk = s0 + row * static_cast<uint32_t>(rs) + (uq >> 3) * 144u;
            d.w[r] = lds128(blk + 16u + k8 * 16u);
            d.m[r] = lds16(blk + 2u * k8);
        } else if constexpr (FMT == kFmtQ4K) {
            const uint32_t sb = uq & 7u;
            const uint32_t blk = s0 + row * static_cast<uint32_t>(rs) + (uq >> 3) * 144u;
            d.w[r] = lds128(blk + 16u + sb * 16u);
            d.m[r] = blk;  // block address: scales are unpacked in slice_math
        }
    }
}

template <int FMT>
__device__ __forceinline__ void slice_load(SliceData& d, uint32_t s0, uint32_t s1, int nq, int rs, const XAddr& xs,
                                           const uint32_t rr[4], int q) {
    slice_load_x<FMT>(d, xs, q);
    slice_load_w<FMT>(d, s0, s1, nq, rs, rr, q);
}

template <int FMT>
__device__ __forceinline__ void slice_math(float a[4], const SliceData& d, uint32_t q) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int dot = dot_nib32_split(d.w[r], d.xa, d.xb);
        if constexpr (FMT == kFmtPreq2 || FMT == kFmtPreq) {
            const float2 sz = half2_bits_to_float2(d.m[r]);  // (scale, zero)
            const float ws = sz.x, wz = sz.y;
            a[r] = __fmaf_rn(small_int_to_float(dot), __fmul_rn(ws, d.xs), a[r]);
            a[r] = __fmaf_rn(-__fmul_rn(wz, ws), d.xss, a[r]);
        } else if constexpr (FMT == kFmtQ4K) {
            // reference Q4_K sub-block (gemv_q4_avx2.cpp:294-329): 6-bit LE bitstream values
            // sb (scale) and sb + 8 (min) of the super-block at d.m[r]
            const uint32_t blk = d.m[r];
            const uint32_t sb = q & 7u;
            const uint32_t dd = lds32(blk);
            const float dsc = half_bits_to_float(dd), dmin = half_bits_to_float(dd >> 16);
            auto get6 = [&](uint32_t idx) -> int {
                const uint32_t bit = idx * 6u, byte = bit >> 3, off = bit & 7u;
                const uint32_t lo = lds8(blk + 4u + byte);
                if (off <= 2) return static_cast<int>((lo >> off) & 0x3Fu);
                return static_cast<int>(((lo >> off) | (lds8(blk + 5u + byte) << (8u - off))) & 0x3Fu);
            };
            const float sub_scale = __fmul_rn(dsc, static_cast<float>(get6(sb)));
            const float sub_min = __fmul_rn(dmin, static_cast<float>(get6(sb + 8u)));
            const float part = __fsub_rn(__fmul_rn(sub_scale, small_int_to_float(dot)),
                                         __fmul_rn(sub_min, small_int_to_float(d.xsi)));
            a[r] = __fmaf_rn(part, d.xs, a[r]);
        } else {
            // symmetric formats: implicit zero 8 (Q4_128, S256)
            const float ws = half_bits_to_float(d.m[r]);
            a[r] = __fmaf_rn(small_int_to_float(dot), __fmul_rn(ws, d.xs), a[r]);
            a[r] = __fmaf_rn(-__fmul_rn(8.0f, ws), d.xss, a[r]);
        }
    }
}

template <int FMT>
__device__ __forceinline__ void band_compute(float a[4], uint32_t s0, uint32_t s1, int K, int rs, const XAddr& xs,
                                             int lane, const uint32_t (&rr)[4], int q0, int q1) {
    const int nq = K >> 5;
#pragma unroll
    for (int r = 0; r < 4; ++r) a[r] = 0.0f;
    // two slices in flight: load both, then do the math
    int q = q0 + lane;
    for (; q + 32 < q1; q += 64) {
        SliceData d0, d1;
        slice_load<FMT>(d0, s0, s1, nq, rs, xs, rr, q);
        slice_load<FMT>(d1, s0, s1, nq, rs, xs, rr, q + 32);
        slice_math<FMT>(a, d0, static_cast<uint32_t>(q));
        slice_math<FMT>(a, d1, static_cast<uint32_t>(q + 32));
    }
    if (q < q1) {
        SliceData d0;
        slice_load<FMT>(d0, s0, s1, nq, rs, xs, rr, q);
        slice_math<FMT>(a, d0, static_cast<uint32_t>(q));
    }
}

// ---------------------------------------------------------------------------
// Exact-mode rows (kFmtPreq2X*): the reference's process_one_row (gemv_preq2_avx2.cpp:216-253) in
// its compiled order, for a unit of LPT bands (4 * LPT rows).  Eight int32 dot lanes per group --
// lane j = elements 4j..4j+3, as pmaddubsw + pmaddwd produce them -- are spread over 8 / LPT
// threads per row, LPT consecutive lanes each; every thread keeps its lanes of the even-group and
// odd-group float accumulators and runs the row's two scalar correction chains.  Per group g, in
// order: combined = ws*xs; corr = (wz*ws)*xsum_scaled; acc[g&1][j] += (float)dot_j * combined;
// corr_sum[g&1] += corr.  Row value = (hsum(acc_even) + hsum(acc_odd)) - (corr_even + corr_odd),
// hsum = ((v0+v4)+(v1+v5)) + ((v2+v6)+(v3+v7)), returned in every thread of the row.
// The activation codes are in lane order (kProA8X / kProRmsA8X): lane j of group g is the word at
// x8 + 32g + 4j with codes [4j, 4j+2, 4j+1, 4j+3], the byte order of the nibble word below.
// ---------------------------------------------------------------------------
// lane words of 4 nibble bytes w (lanes A = bytes 0-1, B = bytes 2-3): bytes [e0, e2, e1, e3]
__device__ __forceinline__ uint32_t nib_lane_lo(uint32_t w) { return (w & 0x0F0Fu) | ((w << 12) & 0x0F0F0000u); }
__device__ __forceinline__ uint32_t nib_lane_hi(uint32_t w) {
    return ((w >> 16) & 0x0F0Fu) | ((w >> 4) & 0x0F0F0000u);
}

// Two byte layouts of a unit of LPT bands (4 * LPT rows):
//   kInter = false: the reference's preq2 bytes as they are -- quant [band][g][4 rows][16 B], meta
//     [row][g][4 B] -- whose meta rows are ng*4 bytes apart, a multiple of 128: the rows of a warp
//     read one bank (used by the standalone exact entry points);
//   kInter = true: the engine's exact layout (k_relayout_exact, pure byte moves at finalize) --
//     quant [g][4*LPT rows][16 B] and meta [g][4*LPT rows][4 B] per unit -- where every group's
//     bytes of all the unit's rows are contiguous: conflict-free loads.
template <int LPT, bool kInter>
__device__ __forceinline__ float rows_exact(const uint8_t* sq, const uint8_t* sm, int K, const uint8_t* x8,
                                            const float* xz, int lane, int half) {
    // the even-group and odd-group chains of a row are independent: threads of a row split by
    // parity first, then by lane sets of LPT lanes
    constexpr int TPR = 16 / LPT;  // threads per row
    constexpr int HT = TPR / 2;    // threads per row and parity
    const int nq = K >> 5;
    const int rho = half * (2 * LPT) + lane / TPR;  // row within the unit
    const int sub = lane % TPR;
    const int par = sub / HT;  // 0: even groups, 1: odd groups
    const int ls = sub % HT;   // this thread's lanes: LPT * ls ..
    const uint8_t* qa;
    const uint8_t* ma;
    int qstride, mstride;
    if constexpr (kInter) {
        qa = sq + rho * 16 + ls * (2 * LPT);
        ma = sm + rho * 4;
        qstride = 64 * LPT;
        mstride = 16 * LPT;
    } else {
        qa = sq + (rho >> 2) * nq * 64 + (rho & 3) * 16 + ls * (2 * LPT);
        ma = sm + rho * nq * 4;
        qstride = 64;
        mstride = 4;
    }
    const uint8_t* xa = x8 + ls * (4 * LPT);
    float acc[LPT];
#pragma unroll
    for (int i = 0; i < LPT; ++i) acc[i] = 0.0f;
    float cor = 0.0f;
    const float kMagic = 12582912.0f;  // 1.5 * 2^23: dp4a accumulates into its bit pattern
#pragma unroll 4
    for (int g = par; g < nq; g += 2) {
        const uint8_t* qg = qa + g * qstride;
        const uint8_t* xg = xa + g * 32;
        uint32_t lw[LPT];  // lane words of nibbles
        uint32_t xw[LPT];  // activation words
        if constexpr (LPT == 1) {
            lw[0] = nib_lane_lo(*reinterpret_cast<const uint16_t*>(qg));
            xw[0] = *reinterpret_cast<const uint32_t*>(xg);
        } else if constexpr (LPT == 2) {
            const uint32_t w = *reinterpret_cast<const uint32_t*>(qg);
            lw[0] = nib_lane_lo(w);
            lw[1] = nib_lane_hi(w);
            const uint2 x2 = *reinterpret_cast<const uint2*>(xg);
            xw[0] = x2.x;
            xw[1] = x2.y;
        } else if constexpr (LPT == 4) {
            const uint2 w = *reinterpret_cast<const uint2*>(qg);
            lw[0] = nib_lane_lo(w.x);
            lw[1] = nib_lane_hi(w.x);
            lw[2] = nib_lane_lo(w.y);
            lw[3] = nib_lane_hi(w.y);
            const uint4 x4 = *reinterpret_cast<const uint4*>(xg);
            xw[0] = x4.x;
            xw[1] = x4.y;
            xw[2] = x4.z;
            xw[3] = x4.w;
        } else {
            const uint4 w = *reinterpret_cast<const uint4*>(qg);
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                lw[2 * i] = nib_lane_lo(ww[i]);
                lw[2 * i + 1] = nib_lane_hi(ww[i]);
            }
            const uint4 xa4 = *reinterpret_cast<const uint4*>(xg), xb4 = *reinterpret_cast<const uint4*>(xg + 16);
            xw[0] = xa4.x;
            xw[1] = xa4.y;
            xw[2] = xa4.z;
            xw[3] = xa4.w;
            xw[4] = xb4.x;
            xw[5] = xb4.y;
            xw[6] = xb4.z;
            xw[7] = xb4.w;
        }
        const float2 sz = half2_bits_to_float2(*reinterpret_cast<const uint32_t*>(ma + g * mstride));  // (ws, wz)
        const float2 xs2 = *reinterpret_cast<const float2*>(xz + 2 * g);  // (xs, xsum_scaled)
        const float comb = __fmul_rn(sz.x, xs2.x);
#pragma unroll
        for (int i = 0; i < LPT; ++i) {
            // (float)dot exactly: |dot| < 2^13, so 0x4B400000 + dot is the float 1.5*2^23 + dot
            const float d = __fsub_rn(__int_as_float(dp4a_us(lw[i], xw[i], 0x4B400000)), kMagic);
            acc[i] = __fadd_rn(acc[i], __fmul_rn(d, comb));
        }
        cor = __fadd_rn(cor, __fmul_rn(__fmul_rn(sz.y, sz.x), xs2.y));
    }
    // hsum over this parity's 8 lanes, held LPT per thread by HT threads
    float hs;
    if constexpr (LPT == 8) {
        hs = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[4]), __fadd_rn(acc[1], acc[5])),
                       __fadd_rn(__fadd_rn(acc[2], acc[6]), __fadd_rn(acc[3], acc[7])));
    } else if constexpr (LPT == 4) {
        float a[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = __fadd_rn(acc[i], __shfl_xor_sync(0xffffffffu, acc[i], 1));
        hs = __fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3]));
    } else if constexpr (LPT == 2) {
        const float a0 = __fadd_rn(acc[0], __shfl_xor_sync(0xffffffffu, acc[0], 2));
        const float a1 = __fadd_rn(acc[1], __shfl_xor_sync(0xffffffffu, acc[1], 2));
        const float b = __fadd_rn(a0, a1);
        hs = __fadd_rn(b, __shfl_xor_sync(0xffffffffu, b, 1));
    } else {
        const float a = __fadd_rn(acc[0], __shfl_xor_sync(0xffffffffu, acc[0], 4));
        const float b = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 1));
        hs = __fadd_rn(b, __shfl_xor_sync(0xffffffffu, b, 2));
    }
    // (hsum(even) + hsum(odd)) - (corr_even + corr_odd): the partner thread holds the other parity
    const float hs2 = __shfl_xor_sync(0xffffffffu, hs, HT);
    const float cor2 = __shfl_xor_sync(0xffffffffu, cor, HT);
    return __fsub_rn(__fadd_rn(hs, hs2), __fadd_rn(cor, cor2));
}

// The exact layout of one preq2 matrix (rows M, ng = K/32 groups) in units of L bands: quant
// [unit][g][4L rows][16 B], meta [unit][g][4L rows][4 B]; rows past M are zero.  Pure byte moves;
// one thread per (unit, group, row).
__global__ void k_relayout_exact(const uint8_t* __restrict__ meta, const uint8_t* __restrict__ quant,
                                 uint8_t* __restrict__ meta_x, uint8_t* __restrict__ quant_x, long long M, int ng,
                                 int L, long long units) {
    const long long R = 4ll * L;
    const long long total = units * ng * R;
    for (long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = t % R;
        const long long ug = t / R;
        const long long g = ug % ng;
        const long long u = ug / ng;
        const long long row = u * R + r;
        uint4 qv = make_uint4(0u, 0u, 0u, 0u);
        uint32_t mv = 0u;
        if (row < M) {
            const long long band = row >> 2;
            qv = *reinterpret_cast<const uint4*>(quant + (band * ng + g) * 64 + (row & 3) * 16);
            mv = *reinterpret_cast<const uint32_t*>(meta + (row * ng + g) * 4);
        }
        *reinterpret_cast<uint4*>(quant_x + t * 16) = qv;
        *reinterpret_cast<uint32_t*>(meta_x + t * 4) = mv;
    }
}

// rotate a lane's four partials back to row order: v[j] = a[(j - rot) & 3]
__device__ __forceinline__ void unrotate(float a[4], int rot) {
    if (rot & 1) {
        const float t = a[3];
        a[3] = a[2];
        a[2] = a[1];
        a[1] = a[0];
        a[0] = t;
    }
    if (rot & 2) {
        float t = a[0];
        a[0] = a[2];
        a[2] = t;
        t = a[1];
        a[1] = a[3];
        a[3] = t;
    }
}

// reduce-scatter of four per-lane values over the warp: returns, in lane l,
// the warp sum of value j = l >> 3 (rows 0..3 land in lanes 0, 8, 16, 24).
__device__ __forceinline__ float reduce4(const float v[4], int lane) {
    const bool hi16 = lane & 16;
    const float s0 = hi16 ? v[0] : v[2];
    const float s1 = hi16 ? v[1] : v[3];
    const float r0 = __shfl_xor_sync(0xffffffffu, s0, 16);
    const float r1 = __shfl_xor_sync(0xffffffffu, s1, 16);
    const float k0 = (hi16 ? v[2] : v[0]) + r0;
    const float k1 = (hi16 ? v[3] : v[1]) + r1;
    const bool hi8 = lane & 8;
    const float r = __shfl_xor_sync(0xffffffffu, hi8 ? k0 : k1, 8);
    float k = (hi8 ? k1 : k0) + r;
    k += __shfl_xor_sync(0xffffffffu, k, 4);
    k += __shfl_xor_sync(0xffffffffu, k, 2);
    k += __shfl_xor_sync(0xffffffffu, k, 1);
    return k;
}

// packed W4A32 row (no activation quantization): y = sum_g dot_f32 * s + b * sum(x_g)
__device__ __forceinline__ float unit_packed(const uint8_t* wrow, const float* srow, const float* brow, int K,
                                             int gs, const XArea& xa, int lane) {
    float acc = 0.0f;
    const int lanes_per_group = gs / 8;  // gs multiple of 8 (checked on host)
    const bool shuffle_ok = (256 % gs) == 0;
    for (int base = 0; base < K; base += 256) {
        const int k = base + lane * 8;
        float d = 0.0f;
        int g = -1;
        if (k < K) {
            const uint32_t w = *reinterpret_cast<const uint32_t*>(wrow + (k >> 1));
            const float4 x0 = *reinterpret_cast<const float4*>(xa.xf + k);
            const float4 x1 = *reinterpret_cast<const float4*>(xa.xf + k + 4);
            d = __fmaf_rn(nibble_to_float(w), x0.x, d);
            d = __fmaf_rn(nibble_to_float(w >> 4), x0.y, d);
            d = __fmaf_rn(nibble_to_float(w >> 8), x0.z, d);
            d = __fmaf_rn(nibble_to_float(w >> 12), x0.w, d);
            d = __fmaf_rn(nibble_to_float(w >> 16), x1.x, d);
            d = __fmaf_rn(nibble_to_float(w >> 20), x1.y, d);
            d = __fmaf_rn(nibble_to_float(w >> 24), x1.z, d);
            d = __fmaf_rn(nibble_to_float(w >> 28), x1.w, d);
            g = k / gs;
        }
        if (shuffle_ok) {
            for (int o = 1; o < lanes_per_group; o <<= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
            if (g >= 0 && (lane % lanes_per_group) == 0) acc += __fmaf_rn(d, srow[g], __fmul_rn(brow[g], xa.sx[g]));
        } else if (g >= 0) {
            acc = __fmaf_rn(d, srow[g], acc);
            if ((k % gs) == 0) acc = __fmaf_rn(brow[g], xa.sx[g], acc);
        }
    }
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
// producer: one thread streams this CTA's units [u0, u1) of one GEMV, chunk by chunk, into
// the ring slots that follow ring position jg (slot = position % S); jg advances past them.
// Returns false when a wait for a free slot gave up (status bit set).
// ---------------------------------------------------------------------------
template <int NS, int NSEG>
__device__ bool produce_chunks(const PipeArgs& pa, long long u0, long long u1, uint8_t* ring, uint32_t slot_bytes,
                               int S, uint64_t* full, uint64_t* empty, int& jg, unsigned int* status, uint64_t pol) {
    const int CU = pa.units_per_chunk;
    const int n_chunks = static_cast<int>((u1 - u0 + CU - 1) / CU);
    int s = jg % S;
    int use = jg / S;
    for (int j = 0; j < n_chunks; ++j) {
        if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) {
            atomicOr(status, kStatusWaitEmpty);
            jg += j;
            return false;
        }
        const long long cb = u0 + static_cast<long long>(j) * CU;
        const long long ce = (cb + CU < u1) ? cb + CU : u1;
        uint8_t* st = ring + static_cast<size_t>(s) * slot_bytes;
        uint32_t tx = 0;
        bool tail = false;
#pragma unroll
        for (int seg = 0; seg < NSEG; ++seg)
#pragma unroll
            for (int i = 0; i < NS; ++i) {
                const Span sp = chunk_span(pa.s[i], cb + seg * pa.pair_unit_off, ce + seg * pa.pair_unit_off);
                tx += static_cast<uint32_t>(sp.a1 - sp.a0);
                // bytes past the stream's last 16-byte boundary: plain loads by this thread
                const long long t0 = sp.a1 > sp.start ? sp.a1 : sp.start;
                uint8_t* region = st + seg * pa.seg_bytes + pa.s[i].region_off;
                for (long long t = t0; t < sp.end; ++t) {
                    region[t - sp.a0] = pa.s[i].base[t];
                    tail = true;
                }
            }
        if (tail) fence_proxy_async_smem();
        mbar_arrive_expect_tx(&full[s], tx);
#pragma unroll
        for (int seg = 0; seg < NSEG; ++seg)
#pragma unroll
            for (int i = 0; i < NS; ++i) {
                const Span sp = chunk_span(pa.s[i], cb + seg * pa.pair_unit_off, ce + seg * pa.pair_unit_off);
                if (sp.a1 > sp.a0)
                    bulk_g2s_stream(st + seg * pa.seg_bytes + pa.s[i].region_off, pa.s[i].base + sp.a0,
                                    static_cast<uint32_t>(sp.a1 - sp.a0), &full[s], pol);
            }
        if (++s == S) {
            s = 0;
            ++use;
        }
    }
    jg += n_chunks;
    return true;
}

// wait for the copies of the last min(S, jg) ring positions: a CTA never exits with copies in flight
__device__ __forceinline__ void drain_ring(uint64_t* full, int S, int jg, unsigned int* status) {
    const int first = jg > S ? jg - S : 0;
    for (int j = first; j < jg; ++j) {
        if (!mbar_wait(&full[j % S], (j / S) & 1)) {
            atomicOr(status, kStatusWaitDrain);
            break;
        }
    }
}

// ---------------------------------------------------------------------------
// consumers: the 16 consumer warps of a CTA take every chunk of this CTA's units [u0, u1)
// from the ring slots that follow position jg, run the band math and the epilogue, release
// the slots, and advance jg past them.  The A8 area (xa / xad) is filled by the caller.
// ---------------------------------------------------------------------------
template <int FMT, int PRO, int EPI, int NT>
__device__ void consume_chunks(const PipeArgs& pa, const GemvArgs& ga, const XArea& xa, const XAddr& xad,
                               uint32_t xa_stride, long long u0, long long u1, uint8_t* ring, uint32_t slot_bytes,
                               int S, uint64_t* full, uint64_t* empty, float* s_part, int* s_cnt, int& jg,
                               float& best_v, int& best_i, TlCtx tl = TlCtx{~0u, 0u, 0u}) {
    using T = FmtTraits<FMT>;
    constexpr int NS = T::kStreams;
    constexpr int NSEG = epi_is_silu(EPI) ? 2 : 1;
    const int lane = threadIdx.x & 31;
    const int cw = threadIdx.x >> 5;
    const int CU = pa.units_per_chunk;
    const int P = pa.k_parts;
    const int IPU = P * NSEG;
    const int n_chunks = static_cast<int>((u1 - u0 + CU - 1) / CU);
    const int K = ga.K;
    const int M = ga.M;
    const int nq = K >> 5;
    const int rot = (FMT == kFmtPreq2) ? ((lane >> 1) & 3) : ((lane >> 2) & 3);
    // this lane's row visiting order within a band (bank-conflict-free 16-byte loads)
    const uint32_t rr_lane[4] = {static_cast<uint32_t>(rot & 3), static_cast<uint32_t>((rot + 1) & 3),
                                 static_cast<uint32_t>((rot + 2) & 3), static_cast<uint32_t>((rot + 3) & 3)};
    int item_base = jg;  // any per-CTA running offset works; the ring position varies per op
    // ring slot and phase of chunk j, advanced incrementally (no division per chunk)
    int s = jg % S;
    int use = jg / S;
    const uint32_t ring_s = smem_u32(ring);
    for (int j = 0; j < n_chunks; ++j) {
        if (!mbar_wait(&full[s], use & 1)) {
            if (lane == 0) atomicOr(ga.status, kStatusWaitFull);
            jg += n_chunks;
            return;
        }
        if (tl.slot != ~0u && threadIdx.x == 0) {
            if (j == 0) tl_put(tl, kTlFirstFull);
            if (j == n_chunks - 1) tl_put(tl, kTlLastFull);
        }
        const long long cb = u0 + static_cast<long long>(j) * CU;
        const int n_units_here = static_cast<int>(((cb + CU < u1) ? cb + CU : u1) - cb);
        uint8_t* st = ring + static_cast<size_t>(s) * slot_bytes;
        const uint32_t st_s = ring_s + static_cast<uint32_t>(s) * slot_bytes;
        uint32_t ub[NSEG][NS];
#pragma unroll
        for (int sg = 0; sg < NSEG; ++sg)
#pragma unroll
            for (int i = 0; i < NS; ++i)
                ub[sg][i] = st_s + sg * pa.seg_bytes + pa.s[i].region_off +
                            chunk_off16(pa.s[i], cb + sg * pa.pair_unit_off);

        const int n_items = n_units_here * IPU;
        // items are dealt round-robin over the whole run of chunks (not from warp 0 in every
        // chunk), so chunks with fewer items than warps still keep every warp busy
        const int it0 = (cw - item_base % kConsumerWarps + kConsumerWarps) % kConsumerWarps;
        item_base += n_items;
        for (int it = it0; it < n_items; it += kConsumerWarps) {
            // k = it / IPU exactly (small integers), without an integer division
            const int k = (IPU == 1) ? it : __float2int_rz(__fmul_rn(static_cast<float>(it) + 0.5f, pa.inv_ipu));
            const int rem = it - k * IPU;
            const int seg = (NSEG == 1 || rem < P) ? 0 : 1;
            const int part = rem - seg * P;
            const long long unit = cb + k;
            if constexpr (FMT == kFmtPacked) {
                const long long ce = cb + n_units_here;
                const Span sp0 = chunk_span(pa.s[0], cb, ce);
                const Span sp1 = chunk_span(pa.s[1], cb, ce);
                const Span sp2 = chunk_span(pa.s[2], cb, ce);
                const float v = unit_packed(
                    st + pa.s[0].region_off + (sp0.start - sp0.a0) + k * pa.s[0].unit_bytes,
                    reinterpret_cast<const float*>(st + pa.s[1].region_off + (sp1.start - sp1.a0) +
                                                   k * pa.s[1].unit_bytes),
                    reinterpret_cast<const float*>(st + pa.s[2].region_off + (sp2.start - sp2.a0) +
                                                   k * pa.s[2].unit_bytes),
                    K, ga.gs, xa, lane);
                if (lane == 0 && unit < M) ga.y[unit] = v;
            } else if constexpr (NT > 1) {
                const int q0 = (P == 1) ? 0 : pa.q_bounds[part];
                const int q1 = (P == 1) ? nq : pa.q_bounds[part + 1];
                const uint32_t p0 = ub[0][0] + static_cast<uint32_t>(k * pa.s[0].unit_bytes);
                uint32_t p1 = 0u;
                if constexpr (NS > 1) p1 = ub[0][NS - 1] + static_cast<uint32_t>(k * pa.s[NS - 1].unit_bytes);
                const uint32_t rr[4] = {static_cast<uint32_t>(rot & 3), static_cast<uint32_t>((rot + 1) & 3),
                                        static_cast<uint32_t>((rot + 2) & 3), static_cast<uint32_t>((rot + 3) & 3)};
                const int ntok = ga.n_tokens;
                float vt[NT];
                // tokens in groups of TG: each slice's weights are loaded once per group
                constexpr int TG = NT < ASDSL_MT_GROUP ? NT : ASDSL_MT_GROUP;
#pragma unroll
                for (int t0 = 0; t0 < NT; t0 += TG) {
                    if (t0 >= ntok) continue;
                    float a4[TG][4];
#pragma unroll
                    for (int tt = 0; tt < TG; ++tt)
#pragma unroll
                        for (int r = 0; r < 4; ++r) a4[tt][r] = 0.0f;
                    for (int q = q0 + lane; q < q1; q += 32) {
                        SliceData d;
                        slice_load_w<FMT>(d, p0, p1, nq, pa.row_bytes, rr, q);
#pragma unroll
                        for (int tt = 0; tt < TG; ++tt) {
                            if (t0 + tt < ntok) {
                                const uint32_t off = static_cast<uint32_t>(t0 + tt) * xa_stride;
                                XAddr xt;
                                xt.x8 = xad.x8 + off;
                                xt.x8b = xad.x8b + off;
                                xt.xs = xad.xs + off;
                                xt.xss = xad.xss + off;
                                xt.xsi = xad.xsi + off;
                                slice_load_x<FMT>(d, xt, q);
                                slice_math<FMT>(a4[tt], d, static_cast<uint32_t>(q));
                            }
                        }
                    }
#pragma unroll
                    for (int tt = 0; tt < TG; ++tt) {
                        if (t0 + tt < NT) {
                            unrotate(a4[tt], rot);
                            vt[t0 + tt] = reduce4(a4[tt], lane);
                        }
                    }
                }
                bool finish = true;
                if (IPU > 1) {
                    const int slot = s * CU + k;
                    if ((lane & 7) == 0) {
#pragma unroll
                        for (int t = 0; t < NT; ++t)
                            if (t < ntok) s_part[((slot * IPU + rem) * NT + t) * 4 + (lane >> 3)] = vt[t];
                    }
                    __syncwarp();
                    int prev = 0;
                    if (lane == 0) {
                        __threadfence_block();
                        prev = atomicAdd(&s_cnt[slot], 1);
                    }
                    prev = __shfl_sync(0xffffffffu, prev, 0);
                    finish = (prev == IPU - 1);
                    if (finish) {
                        __threadfence_block();
#pragma unroll
                        for (int t = 0; t < NT; ++t) {
                            if (t < ntok) {
                                float acc = 0.0f;
                                for (int p2 = 0; p2 < P; ++p2)
                                    acc += s_part[((slot * IPU + p2) * NT + t) * 4 + (lane >> 3)];
                                vt[t] = acc;
                            }
                        }
                        if (lane == 0) s_cnt[slot] = 0;
                    }
                }
                const long long row = unit * 4 + (lane >> 3);
                if (finish && (lane & 7) == 0 && row < M) {
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        if (t < ntok) {
                            const long long o = static_cast<long long>(t) * M + row;
                            if constexpr (EPI == kEpiResid)
                                ga.resid[o] = __fadd_rn(vt[t], __ldcg(ga.resid + o));  // token t's residual row
                            else
                                ga.y[o] = vt[t];
                        }
                    }
                }
            } else {
                const int q0 = (P == 1) ? 0 : pa.q_bounds[part];
                const int q1 = (P == 1) ? nq : pa.q_bounds[part + 1];
                // the residual row is read before the band math (only this unit writes it), so
                // its L2 round trip overlaps the math; every part of a split reads it, the one
                // that finishes the unit uses it
                float res = 0.0f;
                if constexpr (EPI == kEpiResid) {
                    const int rrow = static_cast<int>(unit) * 4 + (lane >> 3);
                    if ((lane & 7) == 0 && rrow < M) res = __ldcg(ga.resid + rrow);
                }
                float a[4];
                // 32-bit offsets: a stage is far below 4 GB
                const uint32_t p0 = (seg == 0 ? ub[0][0] : ub[NSEG - 1][0]) +
                                    static_cast<uint32_t>(k) * static_cast<uint32_t>(pa.s[0].unit_bytes);
                uint32_t p1 = 0u;
                if constexpr (NS > 1)
                    p1 = (seg == 0 ? ub[0][NS - 1] : ub[NSEG - 1][NS - 1]) +
                         static_cast<uint32_t>(k) * static_cast<uint32_t>(pa.s[NS - 1].unit_bytes);
                band_compute<FMT>(a, p0, p1, K, pa.row_bytes, xad, lane, rr_lane, q0, q1);
                unrotate(a, rot);
                const float v = reduce4(a, lane);
                float vrow[NSEG];
                bool finish = true;
                if (IPU > 1) {
                    // deposit this item's row partials; the last item of the unit sums all
                    // of them in a fixed order (deterministic) and runs the epilogue
                    const int slot = s * CU + k;
                    if ((lane & 7) == 0) s_part[(slot * IPU + rem) * 4 + (lane >> 3)] = v;
                    __syncwarp();
                    int prev = 0;
                    if (lane == 0) {
                        __threadfence_block();
                        prev = atomicAdd(&s_cnt[slot], 1);
                    }
                    prev = __shfl_sync(0xffffffffu, prev, 0);
                    finish = (prev == IPU - 1);
                    if (finish) {
                        __threadfence_block();
#pragma unroll
                        for (int sg = 0; sg < NSEG; ++sg) {
                            float acc = 0.0f;
                            for (int p2 = 0; p2 < P; ++p2) acc += s_part[(slot * IPU + sg * P + p2) * 4 + (lane >> 3)];
                            vrow[sg] = acc;
                        }
                        if (lane == 0) s_cnt[slot] = 0;  // re-arm for the stage's next use
                    }
                } else {
                    vrow[0] = v;
                }
                const int row = static_cast<int>(unit) * 4 + (lane >> 3);  // rows are an int (M)
                if (finish && (lane & 7) == 0 && row < M) {
                    if constexpr (EPI == kEpiStore) {
                        ga.y[row] = vrow[0];
                    } else if constexpr (EPI == kEpiResid) {
                        // L2 read (res, above): in a persistent kernel other CTAs wrote neighbouring
                        // rows of this line
                        ga.resid[row] = __fadd_rn(vrow[0], res);
                    } else if constexpr (EPI == kEpiSilu) {
                        ga.h[row] = ref_silu_mul(vrow[0], vrow[NSEG - 1]);

                    } else {
                        if (ga.y) ga.y[row] = vrow[0];
                        argmax_take(best_v, best_i, vrow[0], ga.row_base + static_cast<int>(row));
                    }
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
    jg += n_chunks;
}

// ---------------------------------------------------------------------------
// exact-mode consumers (kFmtPreq2X*): a work item is one half of a unit of LPT bands (2 * LPT
// rows), taken by one warp; the paired SiLU form computes the item's gate rows and then its up rows
// in the same warp, so no partial sums cross warps.  A row's value is written by its first thread.
// ---------------------------------------------------------------------------
template <int FMT, int PRO, int EPI, bool kInter>
__device__ void consume_chunks_x(const PipeArgs& pa, const GemvArgs& ga, const XArea& xa, long long u0, long long u1,
                                 uint8_t* ring, int S, uint64_t* full, uint64_t* empty, int& jg, float& best_v,
                                 int& best_i) {
    constexpr int LPT = exact_lpt(FMT);
    constexpr int TPR = 16 / LPT;  // threads per row (rows_exact)
    constexpr int NSEG = epi_is_silu(EPI) ? 2 : 1;
    const int lane = threadIdx.x & 31;
    const int cw = threadIdx.x >> 5;
    const int CU = pa.units_per_chunk;
    const int n_chunks = static_cast<int>((u1 - u0 + CU - 1) / CU);
    const int K = ga.K;
    const int M = ga.M;
    const uint8_t* x8 = reinterpret_cast<const uint8_t*>(xa.x8);
    const float* xz = xa.xs;  // (scale, xsum_scaled) pairs
    int item_base = jg;
    int s = jg % S;
    int use = jg / S;
    const bool writer = (lane % TPR) == 0;
    for (int j = 0; j < n_chunks; ++j) {
        if (!mbar_wait(&full[s], use & 1)) {
            if (lane == 0) atomicOr(ga.status, kStatusWaitFull);
            jg += n_chunks;
            return;
        }
        const long long cb = u0 + static_cast<long long>(j) * CU;
        const int n_units_here = static_cast<int>(((cb + CU < u1) ? cb + CU : u1) - cb);
        const uint8_t* st = ring + static_cast<size_t>(s) * pa.stage_bytes;
        const uint8_t* ub[NSEG][2];
#pragma unroll
        for (int sg = 0; sg < NSEG; ++sg)
#pragma unroll
            for (int i = 0; i < 2; ++i)
                ub[sg][i] = st + sg * pa.seg_bytes + pa.s[i].region_off + chunk_off16(pa.s[i], cb + sg * pa.pair_unit_off);
        // two items per unit: its first and second half of rows
        const int n_items = 2 * n_units_here;
        const int it0 = (cw - item_base % kConsumerWarps + kConsumerWarps) % kConsumerWarps;
        item_base += n_items;
        for (int it = it0; it < n_items; it += kConsumerWarps) {
            const int un = it >> 1, half = it & 1;
            const long long o0 = static_cast<long long>(un) * pa.s[0].unit_bytes;
            const long long o1 = static_cast<long long>(un) * pa.s[1].unit_bytes;
            const int row = static_cast<int>(cb + un) * (4 * LPT) + half * (2 * LPT) + lane / TPR;
            // the residual row is read before the row math (only this item writes it), so its
            // L2 round trip overlaps the math instead of following it
            float res = 0.0f;
            if constexpr (EPI == kEpiResid)
                if (writer && row < M) res = __ldcg(ga.resid + row);
            const float v = rows_exact<LPT, kInter>(ub[0][0] + o0, ub[0][1] + o1, K, x8, xz, lane, half);
            if constexpr (EPI == kEpiSiluX) {
                const float u =
                    rows_exact<LPT, kInter>(ub[NSEG - 1][0] + o0, ub[NSEG - 1][1] + o1, K, x8, xz, lane, half);
                if (writer && row < M) ga.h[row] = exact_silu_mul(v, u, ga.ex.rcp);
            } else if (writer && row < M) {
                if constexpr (EPI == kEpiStore) {
                    ga.y[row] = v;
                } else if constexpr (EPI == kEpiResid) {
                    ga.resid[row] = __fadd_rn(v, res);
                } else if constexpr (EPI == kEpiArgmax) {
                    if (ga.y) ga.y[row] = v;
                    argmax_take(best_v, best_i, v, ga.row_base + row);
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
    jg += n_chunks;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int FMT, int PRO, int EPI, int NT = 1>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) k_stream_gemv(const PipeArgs pa, const GemvArgs ga) {
    static_assert(NT == 1 || ((EPI == kEpiStore || EPI == kEpiResid) && FMT != kFmtPacked && !is_exact_fmt(FMT)),
                  "multi-token: store or residual epilogue, W4A8 formats, not the exact mode");
    static_assert(is_exact_fmt(FMT) == pro_is_lane_order(PRO), "kFmtPreq2X* pairs with the lane-order prologues");
    static_assert(is_exact_fmt(FMT) || EPI != kEpiSiluX, "kEpiSiluX is the exact mode's epilogue");
    using T = FmtTraits<FMT>;
    constexpr int NS = T::kStreams;
    constexpr int NSEG = epi_is_silu(EPI) ? 2 : 1;
    constexpr bool kF32 = (PRO == kProF32);
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    uint8_t* stages = smem + pa.stage_off;
    const int S = pa.n_stages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    XArea xa = xarea_layout(smem + pa.xarea_off, ga.K, ga.gs, kF32);

    const long long U = pa.n_units;
    const long long u0 = U * blockIdx.x / gridDim.x;
    const long long u1 = U * (blockIdx.x + 1) / gridDim.x;
    const int CU = pa.units_per_chunk;
    const int P = pa.k_parts;
    const int IPU = P * NSEG;  // work items per unit
    // split partials [stage][unit in chunk][item][row] and per-unit arrival counts
    float* s_part = reinterpret_cast<float*>(smem + pa.split_off);
    int* s_cnt = reinterpret_cast<int*>(s_part + S * CU * IPU * 4 * NT);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_mbar_init();
    }
    __shared__ uint32_t s_tl;
    if constexpr (kTimeline)
        if (threadIdx.x == 0) s_tl = tl_slot();
    if (IPU > 1)
        for (int i = threadIdx.x; i < S * CU; i += blockDim.x) s_cnt[i] = 0;
    __syncthreads();
    // let a dependent kernel launch now; it touches our outputs only after its own wait
    grid_launch_dependents();
    const uint32_t tl = kTimeline ? s_tl : ~0u;  // a constant outside the timeline build
    if (threadIdx.x == 0) tl_rec<FMT, PRO, EPI, NT>(tl, kTlStart, ga.tl_id);

    if (warp == kProducerWarp) {
        if (lane != 0) return;
        // weights never depend on the previous kernel: stream them before its completion
        const uint64_t pol = l2_policy_evict_first();
        int jg = 0;
        produce_chunks<NS, NSEG>(pa, u0, u1, stages, pa.stage_bytes, S, full, empty, jg, ga.status, pol);
        tl_rec<FMT, PRO, EPI, NT>(tl, kTlProduced, ga.tl_id);
        drain_ring(full, S, jg, ga.status);
        return;
    }

    // ---------------- consumer warps: every warp takes part of every stage ----------------
    const int cw = warp;
    // (loading the RMSNorm weights into registers before the wait was measured: the decode step
    // got 4 % slower, the registers held across the wait costing more than the load it hid)
    grid_dependency_wait();  // activations / residual written by the previous kernel are visible now
    if (threadIdx.x == 0) tl_rec<FMT, PRO, EPI, NT>(tl, kTlWaited, ga.tl_id);
    if constexpr (EPI == kEpiArgmax) {
        if (ga.xchg_stamps != nullptr && blockIdx.x == 0 && threadIdx.x == 0)
            ga.xchg_stamps[((*ga.xchg_epoch + 1) & ga.xchg_stamp_mask) * 4] = globaltimer_ns();
    }
    constexpr uint32_t tl_code = (static_cast<uint32_t>(FMT) << 4) | (static_cast<uint32_t>(PRO) << 8) |
                                 (static_cast<uint32_t>(EPI) << 12) | (static_cast<uint32_t>(NT) << 16);
    // multi-token: one A8 area per activation row, xa_stride bytes apart
    const uint32_t xa_stride = (NT > 1) ? xarea_layout_bytes(ga.K, ga.gs, false) : 0u;
    if constexpr (NT == 1) {
        run_prologue<PRO>(ga, xa, threadIdx.x, TlCtx{tl, tl_code, ga.tl_id});
    } else {
        token_prologue<PRO>(ga, smem + pa.xarea_off, xa_stride);
    }
    if (threadIdx.x == 0) tl_rec<FMT, PRO, EPI, NT>(tl, kTlPrologue, ga.tl_id);

    XAddr xad;
    xad.x8 = kF32 ? 0u : smem_u32(xa.x8);
    xad.x8b = kF32 ? 0u : xad.x8 + static_cast<uint32_t>(ga.K >> 1);
    xad.xs = kF32 ? 0u : smem_u32(xa.xs);
    xad.xss = kF32 ? 0u : smem_u32(xa.xss);
    xad.xsi = kF32 ? 0u : smem_u32(xa.xsi);
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;

    {
        int jg = 0;
        if constexpr (is_exact_fmt(FMT)) {
            if (ga.exact_inter)
                consume_chunks_x<FMT, PRO, EPI, true>(pa, ga, xa, u0, u1, stages, S, full, empty, jg, best_v, best_i);
            else
                consume_chunks_x<FMT, PRO, EPI, false>(pa, ga, xa, u0, u1, stages, S, full, empty, jg, best_v, best_i);
        } else
            consume_chunks<FMT, PRO, EPI, NT>(pa, ga, xa, xad, xa_stride, u0, u1, stages, pa.stage_bytes, S, full,
                                              empty, s_part, s_cnt, jg, best_v, best_i, TlCtx{tl, tl_code, ga.tl_id});
    }
    if (tl != ~0u) {
        if (threadIdx.x == 0) tl_rec<FMT, PRO, EPI, NT>(tl, kTlConsumed, ga.tl_id);
        consumer_sync();
        if (threadIdx.x == 0) tl_rec<FMT, PRO, EPI, NT>(tl, kTlEnd, ga.tl_id);
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
        __shared__ int s_last;
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
            s_last = (prev == gridDim.x - 1) ? 1 : 0;
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
                float fv = bv;
                int fi = (bi == 0x7fffffff) ? ga.row_base : bi;
                if (ga.xchg_self != nullptr) {
                    // fused all-gather of (max, index): store this rank's word into every rank's
                    // slot (NVLink peer stores), then wait -- bounded -- for all words of this
                    // step and keep the first maximum in rank order (= lowest global index)
                    const int W = ga.xchg_world;
                    const int e = *ga.xchg_epoch + 1;
                    const int par = e & 1;
                    const unsigned long long e8 = static_cast<unsigned long long>(e & 0xFF);
                    const unsigned long long word = static_cast<unsigned long long>(__float_as_uint(fv)) |
                                                    (static_cast<unsigned long long>(fi & 0xFFFFFF) << 32) |
                                                    (e8 << 56);
                    unsigned long long* stamp =
                        ga.xchg_stamps ? ga.xchg_stamps + (e & ga.xchg_stamp_mask) * 4 : nullptr;
                    if (stamp) stamp[1] = globaltimer_ns();
                    // the word carries its own step tag: relaxed stores, no system-scope fence
                    for (int r = 0; r < W; ++r) st_relaxed_sys_u64(ga.xchg_peers[r] + par * W + ga.xchg_rank, word);
                    if (stamp) stamp[2] = globaltimer_ns();
                    float gv = -INFINITY;
                    int gi = fi;
                    bool ok = true;
                    const unsigned long long t0 = globaltimer_ns();
                    for (int r = 0; r < W && ok; ++r) {
                        unsigned long long w = ld_relaxed_sys_u64(ga.xchg_self + par * W + r);
                        while ((w >> 56) != e8) {
                            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                                ok = false;
                                break;
                            }
                            w = ld_relaxed_sys_u64(ga.xchg_self + par * W + r);
                        }
                        if (!ok) break;
                        const float v = __uint_as_float(static_cast<unsigned int>(w));
                        if (r == 0 || v > gv) {
                            gv = v;
                            gi = static_cast<int>((w >> 32) & 0xFFFFFFull);
                        }
                    }
                    if (stamp) stamp[3] = globaltimer_ns();
                    if (ok) {
                        fv = gv;
                        fi = gi;
                    } else {
                        atomicOr(ga.status, kStatusXchgWait);
                    }
                    *ga.xchg_epoch = e;
                }
                *ga.out_val = fv;
                *ga.out_idx = fi;
                *ga.counter = 0u;  // re-arm for the next call
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Q4_128 -> banded device layout (pure byte moves; bit-exact by construction):
//   quant  [nb][K/128][4 rows][64 B nibbles]   scales [nb][K/128][4 rows] fp16
// rows past M in the last band are zero.  One thread per (band, group, row).
// ---------------------------------------------------------------------------
__global__ void k_relayout_q4_128(const uint8_t* __restrict__ blocks, uint8_t* __restrict__ quant,
                                  uint8_t* __restrict__ scales, int M, int K) {
    const int ng = K / 128;
    const long long nb = (M + 3) / 4;
    const long long total = nb * ng * 4;
    for (long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(t & 3);
        const long long bg = t >> 2;
        const int g = static_cast<int>(bg % ng);
        const long long b = bg / ng;
        const long long row = b * 4 + r;
        uint8_t* qd = quant + (bg * 4 + r) * 64;
        uint8_t* sd = scales + (bg * 4 + r) * 2;
        if (row < M) {
            const uint8_t* src = blocks + (row * ng + g) * 66;
            sd[0] = src[0];
            sd[1] = src[1];
            for (int i = 0; i < 64; ++i) qd[i] = src[2 + i];
        } else {
            sd[0] = 0;
            sd[1] = 0;
            for (int i = 0; i < 64; ++i) qd[i] = 0;
        }
    }
}

}  // namespace asdsl
