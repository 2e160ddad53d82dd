// decode_step.cuh -- one persistent kernel per decode step (UnifiedEngine::forward_token,
// asdsl/kernels/native/unified_engine.cpp:1339-1688).
//
// The step is a program of ops executed by one cooperative launch, one CTA per SM:
//   embed -> per layer [qkv, attention, o, gate_up+SiLU, down] -> lm_head + argmax -> advance.
// Every op consumes the previous op's output, so a grid barrier separates consecutive ops.
// The weight streams never depend on activations: each CTA's producer warp walks the whole
// program and keeps streaming the next projections' bands through the CTA's shared-memory
// ring while the consumer warps wait at a barrier, run a prologue or finish a tail.  HBM stays
// busy across op boundaries, and the per-kernel launch / prologue / pipeline-fill cost of a
// 163-kernel chain is paid once per token.
//
// Waits are bounded: ring waits as in the streaming GEMV, grid barriers by the same 2 s
// limit; a CTA that gives up sets a status bit and skips the rest of the program (its
// producer's waits then give up too), so the kernel always ends.
#pragma once

#include "engine_ops.cuh"
#include "gemv_stream.cuh"

namespace asdsl {

enum StepOpType : int { kOpEmbed = 0, kOpGemv = 1, kOpAttn = 2, kOpArgmaxFinal = 3 };

// the GEMV variants of the decode program: format x (prologue, epilogue)
enum StepGemvKind : int {
    kGvStore = 0,   // RMSNorm + A8 prologue, store            (qkv)
    kGvResid = 1,   // A8 prologue, residual += y              (o, down)
    kGvSilu = 2,    // RMSNorm + A8 prologue, SiLU(gate) * up  (gate_up)
    kGvArgmax = 3,  // RMSNorm + A8 prologue, per-CTA argmax   (lm_head)
};

struct StepOp {
    int type;
    int kind;
    int fmt;  // kFmtPreq2 or kFmtQ128B
    int pad;
    PipeArgs pa;
    GemvArgs ga;
    AttnArgs aa;
};

struct StepArgs {
    const StepOp* ops;
    int n_ops;
    int n_slots;
    uint32_t slot_bytes;
    uint32_t xarea_off;  // A8 area (aliased by the attention scratch)
    uint32_t cnt_off;    // K-split arrival counters (zeroed at start, re-armed by finishers)
    uint32_t cnt_bytes;
    uint32_t part_off;   // K-split partials
    uint32_t ring_off;
    // embed / advance
    const void* emb;
    int emb_f16;
    float* resid;
    int H, V;
    DecodeState* st;
    int* seq;
    int max_seq;
    int decode;          // 1: lm_head argmax -> seq[pos+1]; 0: prefill
    float* part_val;     // [gridDim] per-CTA argmax partials
    int* part_idx;
    float* out_val;
    int* out_idx;
    unsigned int* bar;   // [0] arrivals, [1] generation
    unsigned int* status;
    // optional per-op profile (null = off): [op][3] = earliest start over CTAs, latest end of
    // the op's work, latest exit from the barrier after it (globaltimer ns)
    unsigned long long* trace;
};

constexpr unsigned int kStatusGridWait = 32u;  // a grid barrier gave up waiting

__device__ __forceinline__ unsigned int ld_acquire_gpu_u32(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// grid barrier of the consumer warps (the producer warps never take part); returns false on
// timeout.  One counter, one release-add per CTA: CTA 0 adds 2^31 - (grid - 1), the others 1,
// so each barrier adds exactly 2^31 and flips the top bit when the last CTA arrives (the low
// 31 bits return to zero, and the counter needs no reset between barriers or launches).
__device__ bool step_grid_barrier(unsigned int* bar, unsigned int* status, int* s_flag) {
    consumer_sync();
    if (threadIdx.x == 0) {
        int ok = 1;
        const unsigned int inc = (blockIdx.x == 0) ? (0x80000000u - (gridDim.x - 1u)) : 1u;
        unsigned int old;
        asm volatile("atom.add.release.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(bar), "r"(inc) : "memory");
        if (((old + inc) ^ old) & 0x80000000u) {
            // this add completed the barrier
        } else {
            const unsigned long long t0 = globaltimer_ns();
            while (((ld_acquire_gpu_u32(bar) ^ old) & 0x80000000u) == 0u) {
                if (globaltimer_ns() - t0 > kWaitLimitNs) {
                    atomicOr(status, kStatusGridWait);
                    ok = 0;
                    break;
                }
            }
        }
        *s_flag = ok;
    }
    consumer_sync();
    return *s_flag != 0;
}

struct AttnWarpSync {
    __device__ __forceinline__ void operator()() const {
        asm volatile("bar.sync 2, %0;" ::"n"(kAttnWarps * 32) : "memory");
    }
};

// the current op's descriptors, staged in shared memory by the consumer warps at the op's start
// (the inner loops then read them from shared memory, not through global-memory loads that
// every epilogue store would force the compiler to repeat)
__shared__ PipeArgs s_op_pa;
__shared__ GemvArgs s_op_ga;
__shared__ AttnArgs s_op_aa;

template <typename T>
__device__ __forceinline__ void stage_struct(T* dst, const T* src) {
    static_assert(sizeof(T) % 4 == 0, "4-byte multiple");
    const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
    uint32_t* d = reinterpret_cast<uint32_t*>(dst);
    for (int i = threadIdx.x; i < static_cast<int>(sizeof(T) / 4); i += kConsumerThreads) d[i] = __ldg(s + i);
}

// one GEMV op on the consumer side: prologue (coherent activation loads), ring chunks, epilogue
template <int FMT, int PRO, int EPI>
__device__ void step_gemv(const StepOp& op, const StepArgs& A, uint8_t* smem, uint64_t* full, uint64_t* empty,
                          int& jg, float& best_v, int& best_i) {
    (void)op;
    const PipeArgs& pa = s_op_pa;
    const GemvArgs& ga = s_op_ga;
    XArea xa = xarea_layout(smem + A.xarea_off, ga.K, ga.gs, false);
    run_prologue<PRO, true>(ga, xa, threadIdx.x);
    XAddr xad;
    xad.x8 = smem_u32(xa.x8);
    xad.x8b = xad.x8 + static_cast<uint32_t>(ga.K >> 1);
    xad.xs = smem_u32(xa.xs);
    xad.xss = smem_u32(xa.xss);
    xad.xsi = smem_u32(xa.xsi);
    const long long U = pa.n_units;
    const long long u0 = U * blockIdx.x / gridDim.x;
    const long long u1 = U * (blockIdx.x + 1) / gridDim.x;
    const int CU = pa.units_per_chunk;
    constexpr int NSEG = (EPI == kEpiSilu) ? 2 : 1;
    const int IPU = pa.k_parts * NSEG;
    (void)CU;
    (void)IPU;
    float* s_part = reinterpret_cast<float*>(smem + A.part_off);
    int* s_cnt = reinterpret_cast<int*>(smem + A.cnt_off);
    consume_chunks<FMT, PRO, EPI, 1>(pa, ga, xa, xad, 0u, u0, u1, smem + A.ring_off, A.slot_bytes, A.n_slots, full,
                                     empty, s_part, s_cnt, jg, best_v, best_i);
}

template <int FMT>
__device__ void step_gemv_dispatch(const StepOp& op, const StepArgs& A, uint8_t* smem, uint64_t* full,
                                   uint64_t* empty, int& jg, float& best_v, int& best_i) {
    switch (op.kind) {
        case kGvStore: step_gemv<FMT, kProRmsA8, kEpiStore>(op, A, smem, full, empty, jg, best_v, best_i); break;
        case kGvResid: step_gemv<FMT, kProA8, kEpiResid>(op, A, smem, full, empty, jg, best_v, best_i); break;
        case kGvSilu: step_gemv<FMT, kProRmsA8, kEpiSilu>(op, A, smem, full, empty, jg, best_v, best_i); break;
        default: step_gemv<FMT, kProRmsA8, kEpiArgmax>(op, A, smem, full, empty, jg, best_v, best_i); break;
    }
}

__global__ void __launch_bounds__(kThreads, 1) k_decode_step(const StepArgs A) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    __shared__ int s_flag;
    __shared__ int s_pos;
    __shared__ float s_bv[kConsumerWarps];
    __shared__ int s_bi[kConsumerWarps];
    const int S = A.n_slots;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_mbar_init();
        s_pos = __ldcg(&A.st->pos);  // one read per CTA: CTA 0 advances it at the very end
    }
    // K-split arrival counters start at zero (finishers re-arm them after each use)
    for (uint32_t i = threadIdx.x; i < A.cnt_bytes / 4; i += blockDim.x)
        reinterpret_cast<int*>(smem + A.cnt_off)[i] = 0;
    __syncthreads();
    const int pos = s_pos;
    const bool pos_ok = pos >= 0 && pos < A.max_seq;

    if (warp == kProducerWarp) {
        if (lane != 0 || !pos_ok) return;
        const uint64_t pol = l2_policy_evict_first();
        int jg = 0;
        for (int i = 0; i < A.n_ops; ++i) {
            const StepOp& op = A.ops[i];
            if (op.type != kOpGemv) continue;
            const long long U = op.pa.n_units;
            const long long u0 = U * blockIdx.x / gridDim.x;
            const long long u1 = U * (blockIdx.x + 1) / gridDim.x;
            const bool ok = (op.kind == kGvSilu)
                                ? produce_chunks<2, 2>(op.pa, u0, u1, smem + A.ring_off, A.slot_bytes, S, full, empty,
                                                       jg, A.status, pol)
                                : produce_chunks<2, 1>(op.pa, u0, u1, smem + A.ring_off, A.slot_bytes, S, full, empty,
                                                       jg, A.status, pol);
            if (!ok) break;
        }
        drain_ring(full, S, jg, A.status);
        return;
    }

    // ---------------- consumer warps ----------------
    int jg = 0;
    bool alive = pos_ok;
    for (int i = 0; i < A.n_ops && alive; ++i) {
        const StepOp& op = A.ops[i];
        if (A.trace && threadIdx.x == 0) atomicMin(A.trace + 3 * i, globaltimer_ns());
        if (op.type == kOpGemv) {
            stage_struct(&s_op_pa, &op.pa);
            stage_struct(&s_op_ga, &op.ga);
            consumer_sync();
        } else if (op.type == kOpAttn) {
            stage_struct(&s_op_aa, &op.aa);
            consumer_sync();
        }
        if (op.type == kOpEmbed) {
            const int tok = __ldcg(A.seq + pos);
            if (tok >= 0 && tok < A.V) {
                const long long row = static_cast<long long>(tok) * A.H;
                for (int e = blockIdx.x * kConsumerThreads + threadIdx.x; e < A.H; e += gridDim.x * kConsumerThreads)
                    A.resid[e] = A.emb_f16 ? half_bits_to_float(static_cast<const uint16_t*>(A.emb)[row + e])
                                           : static_cast<const float*>(A.emb)[row + e];
            }
        } else if (op.type == kOpGemv) {
            float best_v = -INFINITY;
            int best_i = 0x7fffffff;
            if (op.fmt == kFmtPreq2) step_gemv_dispatch<kFmtPreq2>(op, A, smem, full, empty, jg, best_v, best_i);
            else step_gemv_dispatch<kFmtQ128B>(op, A, smem, full, empty, jg, best_v, best_i);
            if (op.kind == kGvArgmax) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
                    argmax_take(best_v, best_i, ov, oi);
                }
                if (lane == 0) {
                    s_bv[warp] = best_v;
                    s_bi[warp] = best_i;
                }
                consumer_sync();
                if (threadIdx.x == 0) {
                    float bv = s_bv[0];
                    int bi = s_bi[0];
                    for (int w = 1; w < kConsumerWarps; ++w) argmax_take(bv, bi, s_bv[w], s_bi[w]);
                    A.part_val[blockIdx.x] = bv;
                    A.part_idx[blockIdx.x] = bi;
                }
            }
        } else if (op.type == kOpAttn) {
            if (static_cast<int>(blockIdx.x) < op.aa.n_heads && warp < kAttnWarps) {
                AttnSmem& S_attn = *reinterpret_cast<AttnSmem*>(smem + A.xarea_off);
                attention_head<true>(s_op_aa, blockIdx.x, S_attn, threadIdx.x, AttnWarpSync());
            }
        } else if (op.type == kOpArgmaxFinal) {
            if (blockIdx.x == 0 && warp == 0) {
                float bv = -INFINITY;
                int bi = 0x7fffffff;
                for (int b = lane; b < static_cast<int>(gridDim.x); b += 32)
                    argmax_take(bv, bi, __ldcg(A.part_val + b), __ldcg(A.part_idx + b));
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    argmax_take(bv, bi, ov, oi);
                }
                if (lane == 0) {
                    *A.out_val = bv;
                    *A.out_idx = (bi == 0x7fffffff) ? 0 : bi;
                }
            }
            if (A.trace && threadIdx.x == 0) {
                atomicMax(A.trace + 3 * i + 1, globaltimer_ns());
                atomicMax(A.trace + 3 * i + 2, globaltimer_ns());
            }
            continue;  // last op: no barrier after it
        }
        if (A.trace) {
            consumer_sync();
            if (threadIdx.x == 0) atomicMax(A.trace + 3 * i + 1, globaltimer_ns());
        }
        if (i + 1 < A.n_ops) alive = step_grid_barrier(A.bar, A.status, &s_flag);
        if (A.trace && threadIdx.x == 0) atomicMax(A.trace + 3 * i + 2, globaltimer_ns());
    }
    // advance the position (and log the token when decoding); one thread, after all ops
    if (alive && blockIdx.x == 0 && threadIdx.x == 0) {
        if (A.decode) A.seq[pos + 1] = *A.out_idx;
        A.st->pos = pos + 1;
    }
}

}  // namespace asdsl
