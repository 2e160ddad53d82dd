// engine.cuh -- device-resident decode engine behind the C ABI (asdsl_b200_engine_*).
//
// Mirrors UnifiedEngine (asdsl/kernels/native/unified_engine.cpp, .h) for the decode
// path: forward_token :1339-1688, generate :1717-1764, reset_session :1325-1337,
// snapshot_kv / restore_kv / truncate_kv :1285-1307.
//
// One decode step is a fixed kernel sequence on the engine's stream:
//   embed -> per layer [ qkv GEMV (RMSNorm + A8 prologue) -> attention (RoPE, int8 KV
//   write, GQA) -> o GEMV (+= residual) -> gate_up GEMV (RMSNorm + A8 prologue, SiLU*up
//   epilogue) -> down GEMV (+= residual) ] -> lm_head GEMV (RMSNorm + A8, fused argmax)
//   -> advance (seq[pos+1] = argmax, pos += 1).
// The position and the token sequence are device-resident, so the sequence is
// captured once as a CUDA graph ("decode"; "prefill" omits the lm_head) and replayed
// per token without a host round trip; kernels chain with programmatic dependent
// launch so each GEMV's weight stream starts while its predecessor drains.
// Included by asdsl_b200.cu (single translation unit).
#pragma once

#include <algorithm>
#include <vector>

#include "decode_step.cuh"
#include "engine_ops.cuh"

namespace {

struct EngProj {
    int fmt = -1;           // ASDSL_B200_FMT_PREQ2 or ASDSL_B200_FMT_Q4_128_BANDED (device layout)
    uint8_t* w0 = nullptr;  // preq2 meta | banded quant
    uint8_t* w1 = nullptr;  // preq2 quant | banded scales
    int rows = 0, cols = 0;
    int xlpt = 0;  // reference-exact mode: w0 / w1 hold the exact layout in units of xlpt bands
};

// a 2-bit draft-bank projection (QCSD): packed codes [rows][cols/4], fp32 scales and biases
// [rows][cols/32]; null when the layer has none for this projection
struct Q2Proj {
    uint8_t* w = nullptr;
    float* s = nullptr;
    float* b = nullptr;
};

struct EngLayer {
    float* rms_att = nullptr;
    float* rms_ffn = nullptr;
    EngProj p[4];  // qkv, o, gate_up, down
    Q2Proj q2[4];
};

constexpr int kProjQkv = 0, kProjO = 1, kProjGateUp = 2, kProjDown = 3;

}  // namespace

struct asdsl_b200_engine {
    asdsl_b200_engine_config cfg{};
    int device = 0;
    cudaStream_t stream = nullptr;
    std::vector<void*> allocs;
    // globals
    void* embed = nullptr;
    int embed_f16 = 1;
    float* out_norm = nullptr;
    float* cos_t = nullptr;
    float* sin_t = nullptr;
    void* out_proj = nullptr;  // lm_head source (fp16 or fp32), dropped after quantization
    int out_proj_f16 = 1;
    std::vector<EngLayer> layers;
    EngProj lm;
    bool lm_ready = false;
    // activations
    float *resid = nullptr, *qkv = nullptr, *att = nullptr, *h = nullptr, *logits = nullptr;
    // int8 KV cache [layer][pos][kv_head][128] + fp32 scales [layer][pos][kv_head][2]
    int8_t *kq = nullptr, *vq = nullptr;
    float *ks = nullptr, *vs = nullptr;
    long long kv_codes_per_layer = 0, kv_scales_per_layer = 0;
    // decode state
    asdsl::DecodeState* st = nullptr;
    int* seq = nullptr;  // [max_seq + 1]
    float* am_val = nullptr;
    int* am_idx = nullptr;
    uint8_t* am_scratch = nullptr;
    // pinned host staging
    int* h_stage = nullptr;  // [4]: pos, token, argmax, status
    cudaGraphExec_t g_decode = nullptr, g_prefill = nullptr;
    // long-cache variants (max_seq_len > 256): attention split over position chunks (256 fast, 128
    // reference-exact); replayed for steps at positions >= 256, where the host-side position
    // mirror says the cache is long
    cudaGraphExec_t g_decode_long = nullptr, g_prefill_long = nullptr;
    bool capture_long = false;
    int host_pos = 0;  // the device position as the host last set and advanced it
    bool finalized = false;
    // per-op kernel chain (default; measured faster on B200) or the persistent decode-step kernel
    int persistent = 0;
    // reference-exact numerics (asdsl_b200_engine_set_numerics): every op in the reference's
    // compiled operation order, with the host CPU's RSQRTSS / RCPPS / expf tables
    int exact = 0;
    asdsl::ExactTabs ex{};
    float inv_sqrt_d = 0.0f;  // 1/sqrt(head_dim) as the reference computes it (RSQRTSS + Newton)
    asdsl::StepOp* d_prog[2] = {nullptr, nullptr};  // [0] prefill, [1] decode
    asdsl::StepArgs prog_args[2] = {};
    uint32_t prog_smem = 0;
    unsigned int* grid_bar = nullptr;
    float* part_val = nullptr;
    int* part_idx = nullptr;
    int kv_seq_len = 0;
    std::vector<int> snapshots;
    // verify (n tokens, all logits): device copy of the tokens and a grow-only logits block
    int* verify_tok = nullptr;          // [max_seq]
    float* verify_logits = nullptr;     // [verify_rows][vocab]
    int verify_rows = 0;
    // batched forward: activation blocks of batch_rows tokens (row t = token t), allocated on first use
    int batch_rows = 0;
    float *b_resid = nullptr, *b_qkv = nullptr, *b_att = nullptr, *b_gu = nullptr, *b_h = nullptr;
    // sharded decode across the GPUs of one box (asdsl_b200_engine_set_shard): this rank holds
    // intermediate_size gate/up rows and down columns of every layer and lm_rows lm_head rows
    // from lm_row_base; the down partials are summed by the peer all-reduce, the argmax by the
    // in-kernel exchange.  Null exchanges = single GPU.
    asdsl_b200_vxchg* vx = nullptr;
    asdsl_b200_xchg* xg = nullptr;
    int lm_rows = 0;  // 0 = vocab_size
    int lm_row_base = 0;
    float* part = nullptr;  // [hidden] this rank's down partial
    // split-KV decode attention (max_seq_len > one chunk): partials [heads][chunks][stride] and
    // per-head arrival counters
    float* attn_part = nullptr;
    unsigned int* attn_cnt = nullptr;
    int attn_chunks = 0;
    asdsl::AttnXSplit xsplit{};  // reference-exact split attention scratch
    // draft steps (forward_token_draft, unified_engine.cpp:1790-1802): layers in `skip` are left
    // out, and with draft_q2 the layers' 2-bit projections replace the 4-bit ones; the step graphs
    // are captured per (q2, long cache) on first use and dropped when the mask or the bank changes
    bool skip[64] = {};
    bool draft_skip = false, draft_q2 = false;  // set while a draft step is enqueued
    cudaGraphExec_t g_draft[4] = {nullptr, nullptr, nullptr, nullptr};
    float* xn = nullptr;  // [hidden] RMSNorm output feeding a 2-bit projection
    float* gu = nullptr;  // [2 * intermediate] 2-bit gate_up output
};

namespace {

// rows of the lm_head this engine holds (all of them unless sharded)
inline int eng_lm_rows(const asdsl_b200_engine* e) { return e->lm_rows > 0 ? e->lm_rows : e->cfg.vocab_size; }

using asdsl::kEcuda;
using asdsl::kEinval;
using asdsl::kErange;
using asdsl::kEtimeout;
using asdsl::kOk;
using asdsl::set_error;

__global__ void k_silu_rows(const float* __restrict__ gu, float* __restrict__ h, int I, int n);

// out = (x * inv) * w, inv = 1/sqrt(mean(x^2) + eps): the fp32 RMSNorm feeding a draft step's 2-bit
// projection (rmsnorm_f32, unified_engine.cpp:499-524; one CTA, block reduction)
__global__ void __launch_bounds__(256) k_rmsnorm_f32(const float* __restrict__ x, const float* __restrict__ w,
                                                     float* __restrict__ out, int n, float eps) {
    __shared__ float red[8];
    grid_dependency_wait();
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += 256) ss = __fmaf_rn(x[i], x[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) tot = __fadd_rn(tot, red[k]);
    const float inv = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(tot, static_cast<float>(n)), eps));
    for (int i = threadIdx.x; i < n; i += 256) out[i] = __fmul_rn(__fmul_rn(x[i], inv), w[i]);
}

template <typename T>
int eng_alloc(asdsl_b200_engine* e, T** p, size_t bytes) {
    void* q = nullptr;
    if (bytes == 0) bytes = 16;
    const cudaError_t rc = cudaMalloc(&q, bytes);
    if (rc != cudaSuccess)
        return set_error(asdsl::kEnomem, std::string("engine: cudaMalloc of ") + std::to_string(bytes) +
                                             " bytes failed: " + cudaGetErrorString(rc));
    e->allocs.push_back(q);
    *p = static_cast<T*>(q);
    return kOk;
}

void eng_free(asdsl_b200_engine* e, void* p) {
    if (!p) return;
    for (auto& q : e->allocs)
        if (q == p) {
            cudaFree(q);
            q = nullptr;
        }
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

void proj_shape(const asdsl_b200_engine_config& c, int which, int* rows, int* cols) {
    const int qd = c.num_heads * c.head_dim, kvd = c.num_kv_heads * c.head_dim;
    switch (which) {
        case kProjQkv: *rows = qd + 2 * kvd; *cols = c.hidden_size; break;
        case kProjO: *rows = c.hidden_size; *cols = qd; break;
        case kProjGateUp: *rows = 2 * c.intermediate_size; *cols = c.hidden_size; break;
        default: *rows = c.hidden_size; *cols = c.intermediate_size; break;
    }
}

// one GEMV of the decode step, with the prologue / epilogue its position needs
template <int PRO, int EPI>
int eng_gemv(const EngProj& p, GemvArgs ga, long long pair_off_rows, cudaStream_t s) {
    StreamIn in[2];
    const long long M = pair_off_rows > 0 ? pair_off_rows : p.rows;
    const long long nb = (M + 3) / 4;
    if (p.fmt == ASDSL_B200_FMT_PREQ2) {
        preq2_streams(in, p.w0, p.w1, p.rows, p.cols);
        ga.gs = 32;
        return launch_stream_gemv<kFmtPreq2, PRO, EPI>(in, 2, nb, pair_off_rows > 0 ? nb : 0, ga, s);
    }
    q128b_streams(in, p.w0, p.w1, p.rows, p.cols);
    ga.gs = 128;
    return launch_stream_gemv<kFmtQ128B, PRO, EPI>(in, 2, nb, pair_off_rows > 0 ? nb : 0, ga, s);
}

// the same GEMV in the reference-exact mode (preq2 weights only; checked at finalize)
template <int PRO, int EPI>
int eng_gemv_x(const asdsl_b200_engine* e, const EngProj& p, GemvArgs ga, long long pair_off_rows, cudaStream_t s) {
    ga.ex = e->ex;
    return launch_exact_gemv<PRO, EPI>(p.w0, p.w1, p.rows, pair_off_rows, ga, s, p.xlpt);
}

int launch_small(const void* fn, dim3 grid, dim3 block, void** args, cudaStream_t s, bool pdl,
                 unsigned dyn_smem = 0) {
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = s;
    cfg.dynamicSmemBytes = dyn_smem;
    cudaLaunchAttribute attr[1];
    if (pdl && launch_policy().pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    ASDSL_CUDA(cudaLaunchKernelExC(&cfg, fn, args));
    return kOk;
}

// ---------------------------------------------------------------------------
// persistent decode-step program (csrc/decode_step.cuh)
// ---------------------------------------------------------------------------
constexpr uint32_t kStepSlotBytes = 40 * 1024;
constexpr uint32_t kStepSmemMax = 227 * 1024;

int eng_gemv_op(const EngProj& p, int kind, const GemvArgs& ga, long long pair_rows, int grid, uint32_t slot,
                int n_slots, asdsl::StepOp& op, uint32_t* part_b, uint32_t* cnt_b) {
    std::memset(&op, 0, sizeof(op));
    op.type = asdsl::kOpGemv;
    op.kind = kind;
    StreamIn in[2];
    const long long M = pair_rows > 0 ? pair_rows : p.rows;
    const long long nb = (M + 3) / 4;
    op.ga = ga;
    op.ga.status = device_status_ptr();
    if (p.fmt == ASDSL_B200_FMT_PREQ2) {
        preq2_streams(in, p.w0, p.w1, p.rows, p.cols);
        op.fmt = kFmtPreq2;
        op.ga.gs = 32;
    } else {
        q128b_streams(in, p.w0, p.w1, p.rows, p.cols);
        op.fmt = kFmtQ128B;
        op.ga.gs = 128;
    }
    op.ga.n_tokens = 1;
    return plan_ring_gemv(in, 2, nb, pair_rows > 0 ? nb : 0, p.cols, grid, slot, n_slots, 0, op.pa, part_b, cnt_b);
}

int eng_build_program(asdsl_b200_engine* e, bool with_lm) {
    const asdsl_b200_engine_config& c = e->cfg;
    const int grid = sm_count();
    if (grid < c.num_heads) return set_error(kEinval, "engine: fewer SMs than attention heads");
    const int H = c.hidden_size;
    // shared memory: barriers | A8 area / attention scratch | K-split counters | partials | ring
    const uint32_t xbytes = round_up(std::max<uint32_t>(xarea_layout_bytes(std::max(H, std::max(c.intermediate_size,
                                                                     c.num_heads * c.head_dim)), 32, false),
                                                        static_cast<uint32_t>(sizeof(asdsl::AttnSmem))), 128);
    std::vector<asdsl::StepOp> ops;
    uint32_t part_max = 0, cnt_max = 0;
    // the ring gets what the fixed regions leave; the split regions are sized after planning,
    // so plan with a conservative slot count first, then check the total
    const uint32_t fixed = kBarBytes + xbytes + 8 * 1024;  // 8 KB reserve for the split regions
    int n_slots = static_cast<int>((kStepSmemMax - 2048 - fixed) / kStepSlotBytes);
    if (n_slots > kMaxStages) n_slots = kMaxStages;
    if (n_slots < 2) return set_error(kEinval, "engine: no room for the decode-step ring");
    auto add_gemv = [&](const EngProj& p, int kind, const GemvArgs& ga, long long pair_rows) -> int {
        asdsl::StepOp op;
        uint32_t pb = 0, cb = 0;
        if (int rc = eng_gemv_op(p, kind, ga, pair_rows, grid, kStepSlotBytes, n_slots, op, &pb, &cb)) return rc;
        part_max = std::max(part_max, pb);
        cnt_max = std::max(cnt_max, cb);
        ops.push_back(op);
        return kOk;
    };
    {
        asdsl::StepOp op;
        std::memset(&op, 0, sizeof(op));
        op.type = asdsl::kOpEmbed;
        ops.push_back(op);
    }
    for (int l = 0; l < c.num_layers; ++l) {
        const EngLayer& L = e->layers[l];
        GemvArgs ga = base_args(L.p[kProjQkv].rows, H, 32);
        ga.x = e->resid;
        ga.norm_w = L.rms_att;
        ga.eps = c.rms_norm_eps;
        ga.y = e->qkv;
        if (int rc = add_gemv(L.p[kProjQkv], asdsl::kGvStore, ga, 0)) return rc;
        {
            asdsl::StepOp op;
            std::memset(&op, 0, sizeof(op));
            op.type = asdsl::kOpAttn;
            op.aa.qkv = e->qkv;
            op.aa.out = e->att;
            op.aa.kq = e->kq + l * e->kv_codes_per_layer;
            op.aa.vq = e->vq + l * e->kv_codes_per_layer;
            op.aa.ks = e->ks + l * e->kv_scales_per_layer;
            op.aa.vs = e->vs + l * e->kv_scales_per_layer;
            op.aa.cos_t = e->cos_t;
            op.aa.sin_t = e->sin_t;
            op.aa.st = e->st;
            op.aa.n_heads = c.num_heads;
            op.aa.n_kv = c.num_kv_heads;
            op.aa.rot = c.rotary_dim;
            op.aa.max_seq = c.max_seq_len;
            ops.push_back(op);
        }
        ga = base_args(H, L.p[kProjO].cols, 32);
        ga.x = e->att;
        ga.resid = e->resid;
        if (int rc = add_gemv(L.p[kProjO], asdsl::kGvResid, ga, 0)) return rc;
        ga = base_args(c.intermediate_size, H, 32);
        ga.x = e->resid;
        ga.norm_w = L.rms_ffn;
        ga.eps = c.rms_norm_eps;
        ga.h = e->h;
        if (int rc = add_gemv(L.p[kProjGateUp], asdsl::kGvSilu, ga, c.intermediate_size)) return rc;
        ga = base_args(H, c.intermediate_size, 32);
        ga.x = e->h;
        ga.resid = e->resid;
        if (int rc = add_gemv(L.p[kProjDown], asdsl::kGvResid, ga, 0)) return rc;
    }
    if (with_lm) {
        GemvArgs ga = base_args(c.vocab_size, H, 32);
        ga.x = e->resid;
        ga.norm_w = e->out_norm;
        ga.eps = c.rms_norm_eps;
        ga.y = e->logits;
        if (int rc = add_gemv(e->lm, asdsl::kGvArgmax, ga, 0)) return rc;
        asdsl::StepOp op;
        std::memset(&op, 0, sizeof(op));
        op.type = asdsl::kOpArgmaxFinal;
        ops.push_back(op);
    }
    const uint32_t cnt_off = kBarBytes + xbytes;
    const uint32_t part_off = cnt_off + round_up(cnt_max, 128);
    const uint32_t ring_off = round_up(part_off + part_max, 128);
    const uint32_t smem = ring_off + static_cast<uint32_t>(n_slots) * kStepSlotBytes;
    if (smem > kStepSmemMax - 2048) return set_error(kEinval, "engine: decode-step shared memory over budget");
    const int idx = with_lm ? 1 : 0;
    if (e->d_prog[idx]) {
        cudaFree(e->d_prog[idx]);
        e->d_prog[idx] = nullptr;
    }
    ASDSL_CUDA(cudaMalloc(reinterpret_cast<void**>(&e->d_prog[idx]), ops.size() * sizeof(asdsl::StepOp)));
    ASDSL_CUDA(cudaMemcpy(e->d_prog[idx], ops.data(), ops.size() * sizeof(asdsl::StepOp), cudaMemcpyHostToDevice));
    asdsl::StepArgs& A = e->prog_args[idx];
    std::memset(&A, 0, sizeof(A));
    A.ops = e->d_prog[idx];
    A.n_ops = static_cast<int>(ops.size());
    A.n_slots = n_slots;
    A.slot_bytes = kStepSlotBytes;
    A.xarea_off = kBarBytes;
    A.cnt_off = cnt_off;
    A.cnt_bytes = round_up(cnt_max, 128);
    A.part_off = part_off;
    A.ring_off = ring_off;
    A.emb = e->embed;
    A.emb_f16 = e->embed_f16;
    A.resid = e->resid;
    A.H = H;
    A.V = c.vocab_size;
    A.st = e->st;
    A.seq = e->seq;
    A.max_seq = c.max_seq_len;
    A.decode = with_lm ? 1 : 0;
    A.part_val = e->part_val;
    A.part_idx = e->part_idx;
    A.out_val = e->am_val;
    A.out_idx = e->am_idx;
    A.bar = e->grid_bar;
    A.status = device_status_ptr();
    e->prog_smem = std::max(e->prog_smem, smem);
    return kOk;
}

int eng_launch_program(asdsl_b200_engine* e, bool with_lm) {
    const asdsl::StepArgs& A = e->prog_args[with_lm ? 1 : 0];
    {
        static std::mutex mu;
        static uint32_t configured[64] = {0};
        int dev = 0;
        cudaGetDevice(&dev);
        std::lock_guard<std::mutex> lk(mu);
        if (dev >= 0 && dev < 64 && configured[dev] < e->prog_smem) {
            ASDSL_CUDA(cudaFuncSetAttribute(asdsl::k_decode_step, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(e->prog_smem)));
            configured[dev] = e->prog_smem;
        }
    }
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(static_cast<unsigned>(sm_count()));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = e->prog_smem;
    cfg.stream = e->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ASDSL_CUDA(cudaLaunchKernelEx(&cfg, asdsl::k_decode_step, A));
    return kOk;
}

// enqueue one forward step (token seq[pos] at st->pos) on e->stream
// one 2-bit draft-bank GEMV (k_gemv_q2, packed); accumulate: y += W x (the residual add)
int eng_q2_gemv(const Q2Proj& q, const float* x, float* y, int M, int K, bool accumulate, cudaStream_t s) {
    const size_t smem = 4ull * (K + K / 32);
    const unsigned grid = static_cast<unsigned>(std::min<long long>((M + asdsl::kQ2Warps - 1) / asdsl::kQ2Warps,
                                                                    sm_count() * 2ll));
    asdsl::k_gemv_q2<true><<<grid, asdsl::kQ2Warps * 32, smem, s>>>(q.w, x, q.s, q.b, y, M, K, 32, accumulate ? 1 : 0);
    ASDSL_CUDA(cudaGetLastError());
    return kOk;
}

int eng_enqueue_step(asdsl_b200_engine* e, bool with_lm) {
    if (e->persistent) return eng_launch_program(e, with_lm);
    const asdsl_b200_engine_config& c = e->cfg;
    cudaStream_t s = e->stream;
    const int H = c.hidden_size;
    {
        const int blocks = (H + 255) / 256;
        if (e->embed_f16) {
            const uint16_t* emb = static_cast<const uint16_t*>(e->embed);
            void* args[] = {&emb, &e->resid, &e->st, &e->seq, const_cast<int*>(&c.hidden_size),
                            const_cast<int*>(&c.vocab_size), const_cast<int*>(&c.max_seq_len)};
            if (int rc = launch_small(reinterpret_cast<const void*>(&k_embed<uint16_t>), dim3(blocks), dim3(256),
                                      args, s, false))
                return rc;
        } else {
            const float* emb = static_cast<const float*>(e->embed);
            void* args[] = {&emb, &e->resid, &e->st, &e->seq, const_cast<int*>(&c.hidden_size),
                            const_cast<int*>(&c.vocab_size), const_cast<int*>(&c.max_seq_len)};
            if (int rc = launch_small(reinterpret_cast<const void*>(&k_embed<float>), dim3(blocks), dim3(256), args,
                                      s, false))
                return rc;
        }
    }
    for (int l = 0; l < c.num_layers; ++l) {
        // a draft step leaves the masked layers out (their KV is not written either)
        if (e->draft_skip && l < 64 && e->skip[l]) continue;
        const EngLayer& L = e->layers[l];
        const bool q2 = e->draft_q2;
        const int qkv_rows = L.p[kProjQkv].rows;
        // qkv = W_qkv . A8(RMSNorm(resid) * rms_att)  (draft bank: W2_qkv . RMSNorm(resid) in fp32)
        if (q2 && L.q2[kProjQkv].w) {
            k_rmsnorm_f32<<<1, 256, 0, s>>>(e->resid, L.rms_att, e->xn, H, c.rms_norm_eps);
            if (int rc = eng_q2_gemv(L.q2[kProjQkv], e->xn, e->qkv, qkv_rows, H, false, s)) return rc;
        } else {
            GemvArgs ga = base_args(L.p[kProjQkv].rows, H, 32);
            ga.x = e->resid;
            ga.norm_w = L.rms_att;
            ga.eps = c.rms_norm_eps;
            ga.y = e->qkv;
            if (int rc = e->exact ? eng_gemv_x<kProRmsA8X, kEpiStore>(e, L.p[kProjQkv], ga, 0, s)
                                  : eng_gemv<kProRmsA8, kEpiStore>(L.p[kProjQkv], ga, 0, s))
                return rc;
        }
        // attention (RoPE, KV write, GQA) -> att
        {
            asdsl::AttnArgs aa;
            aa.qkv = e->qkv;
            aa.out = e->att;
            aa.kq = e->kq + l * e->kv_codes_per_layer;
            aa.vq = e->vq + l * e->kv_codes_per_layer;
            aa.ks = e->ks + l * e->kv_scales_per_layer;
            aa.vs = e->vs + l * e->kv_scales_per_layer;
            aa.cos_t = e->cos_t;
            aa.sin_t = e->sin_t;
            aa.st = e->st;
            aa.n_heads = c.num_heads;
            aa.n_kv = c.num_kv_heads;
            aa.rot = c.rotary_dim;
            aa.max_seq = c.max_seq_len;
            if (e->exact && e->capture_long) {
                // long cache: scores and tile maxima per (head, chunk), then the tile sums and the
                // in-order merge (bitwise the single-CTA kernel's result)
                const dim3 grid(c.num_heads, (c.max_seq_len + asdsl::kAttnXChunk - 1) / asdsl::kAttnXChunk);
                void* a1[] = {&aa, &e->ex, &e->inv_sqrt_d, &e->xsplit};
                if (int rc = launch_small(reinterpret_cast<const void*>(&asdsl::k_attention_exact_scores), grid,
                                          dim3(asdsl::kAttnXThreads), a1, s, true))
                    return rc;
                void* a2[] = {&aa, &e->ex, &e->xsplit};
                if (int rc = launch_small(reinterpret_cast<const void*>(&asdsl::k_attention_exact_sums), grid,
                                          dim3(asdsl::kAttnXThreads), a2, s, true))
                    return rc;
            } else if (e->exact) {
                void* args[] = {&aa, &e->ex, &e->inv_sqrt_d};
                if (int rc = launch_small(reinterpret_cast<const void*>(&asdsl::k_attention_exact), dim3(c.num_heads),
                                          dim3(asdsl::kAttnXThreads), args, s, true,
                                          asdsl::attn_x_layout(c.max_seq_len).total))
                    return rc;
            } else if (e->capture_long && e->attn_chunks > 1) {
                // long cache: heads x position chunks, partials merged in chunk order
                aa.part = e->attn_part;
                aa.cnt = e->attn_cnt;
                void* args[] = {&aa};
                if (int rc = launch_small(reinterpret_cast<const void*>(&asdsl::k_attention_split),
                                          dim3(c.num_heads, e->attn_chunks), dim3(asdsl::kAttnWarps * 32), args, s,
                                          true))
                    return rc;
            } else {
                void* args[] = {&aa};
                if (int rc = launch_small(reinterpret_cast<const void*>(&asdsl::k_attention), dim3(c.num_heads),
                                          dim3(asdsl::kAttnWarps * 32), args, s, true))
                    return rc;
            }
        }
        // resid += W_o . A8(att)
        if (q2 && L.q2[kProjO].w) {
            if (int rc = eng_q2_gemv(L.q2[kProjO], e->att, e->resid, H, L.p[kProjO].cols, true, s)) return rc;
        } else {
            GemvArgs ga = base_args(H, L.p[kProjO].cols, 32);
            ga.x = e->att;
            ga.resid = e->resid;
            if (int rc = e->exact ? eng_gemv_x<kProA8X, kEpiResid>(e, L.p[kProjO], ga, 0, s)
                                  : eng_gemv<kProA8, kEpiResid>(L.p[kProjO], ga, 0, s))
                return rc;
        }
        // h = silu(gate) * up, gate_up = W_gu . A8(RMSNorm(resid) * rms_ffn)
        if (q2 && L.q2[kProjGateUp].w) {
            k_rmsnorm_f32<<<1, 256, 0, s>>>(e->resid, L.rms_ffn, e->xn, H, c.rms_norm_eps);
            if (int rc = eng_q2_gemv(L.q2[kProjGateUp], e->xn, e->gu, 2 * c.intermediate_size, H, false, s)) return rc;
            k_silu_rows<<<static_cast<unsigned>((c.intermediate_size + 255) / 256), 256, 0, s>>>(e->gu, e->h,
                                                                                                 c.intermediate_size, 1);
            ASDSL_CUDA(cudaGetLastError());
        } else {
            GemvArgs ga = base_args(c.intermediate_size, H, 32);
            ga.x = e->resid;
            ga.norm_w = L.rms_ffn;
            ga.eps = c.rms_norm_eps;
            ga.h = e->h;
            if (int rc = e->exact ? eng_gemv_x<kProRmsA8X, kEpiSiluX>(e, L.p[kProjGateUp], ga, c.intermediate_size, s)
                                  : eng_gemv<kProRmsA8, kEpiSilu>(L.p[kProjGateUp], ga, c.intermediate_size, s))
                return rc;
        }
        // resid += W_down . A8(h); sharded: this rank's partial, then the peer all-reduce
        // (every rank's partial summed in rank order, plus the residual)
        if (q2 && L.q2[kProjDown].w) {
            if (int rc = eng_q2_gemv(L.q2[kProjDown], e->h, e->resid, H, c.intermediate_size, true, s)) return rc;
        } else if (e->vx) {
            GemvArgs ga = base_args(H, c.intermediate_size, 32);
            ga.x = e->h;
            ga.y = e->part;
            if (int rc = eng_gemv<kProA8, kEpiStore>(L.p[kProjDown], ga, 0, s)) return rc;
            if (int rc = asdsl_b200_allreduce_peer(e->vx, e->part, e->resid, e->resid, H, s)) return rc;
        } else {
            GemvArgs ga = base_args(H, c.intermediate_size, 32);
            ga.x = e->h;
            ga.resid = e->resid;
            if (int rc = e->exact ? eng_gemv_x<kProA8X, kEpiResid>(e, L.p[kProjDown], ga, 0, s)
                                  : eng_gemv<kProA8, kEpiResid>(L.p[kProjDown], ga, 0, s))
                return rc;
        }
    }
    if (with_lm) {
        GemvArgs ga = base_args(eng_lm_rows(e), H, 32);
        ga.x = e->resid;
        ga.norm_w = e->out_norm;
        ga.eps = c.rms_norm_eps;
        ga.y = e->logits;
        ga.counter = reinterpret_cast<unsigned int*>(e->am_scratch);
        ga.part_val = reinterpret_cast<float*>(e->am_scratch + 256);
        ga.part_idx = reinterpret_cast<int*>(e->am_scratch + 256 + 4 * 1024);
        ga.out_val = e->am_val;
        ga.out_idx = e->am_idx;
        ga.row_base = e->lm_row_base;
        if (e->xg) {
            // the global first maximum: this rank's (max, index) word exchanged inside the kernel
            ga.xchg_peers = e->xg->peer_table;
            ga.xchg_self = e->xg->slots;
            ga.xchg_epoch = e->xg->epoch;
            ga.xchg_world = e->xg->world;
            ga.xchg_rank = e->xg->rank;
        }
        if (int rc = e->exact ? eng_gemv_x<kProRmsA8X, kEpiArgmax>(e, e->lm, ga, 0, s)
                              : eng_gemv<kProRmsA8, kEpiArgmax>(e->lm, ga, 0, s))
            return rc;
        void* args[] = {&e->st, &e->seq, &e->am_idx, const_cast<int*>(&c.max_seq_len)};
        if (int rc = launch_small(reinterpret_cast<const void*>(&asdsl::k_advance_decode), dim3(1), dim3(32), args, s,
                                  true))
            return rc;
    } else {
        void* args[] = {&e->st, const_cast<int*>(&c.max_seq_len)};
        if (int rc = launch_small(reinterpret_cast<const void*>(&asdsl::k_advance_prefill), dim3(1), dim3(32), args,
                                  s, true))
            return rc;
    }
    return kOk;
}

int eng_capture(asdsl_b200_engine* e, bool with_lm, cudaGraphExec_t* out) {
    cudaGraph_t g = nullptr;
    ASDSL_CUDA(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    const int rc = eng_enqueue_step(e, with_lm);
    const cudaError_t ec = cudaStreamEndCapture(e->stream, &g);
    if (rc != kOk) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    ASDSL_CUDA(ec);
    const cudaError_t ei = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    ASDSL_CUDA(ei);
    return kOk;
}

// set pos (and seq[pos] = token when token >= 0) from the pinned stage, stream-ordered
int eng_set_pos(asdsl_b200_engine* e, int pos, int token) {
    ASDSL_CUDA(cudaStreamSynchronize(e->stream));  // the pinned stage may still be read by a prior copy
    e->h_stage[0] = pos;
    e->h_stage[1] = token;
    e->host_pos = pos;
    ASDSL_CUDA(cudaMemcpyAsync(&e->st->pos, &e->h_stage[0], sizeof(int), cudaMemcpyHostToDevice, e->stream));
    if (token >= 0)
        ASDSL_CUDA(cudaMemcpyAsync(e->seq + pos, &e->h_stage[1], sizeof(int), cudaMemcpyHostToDevice, e->stream));
    return kOk;
}

// replay one step graph (decode: with the lm_head and argmax), the long-cache variant for a step at
// position >= 256; the host mirror advances as k_advance_* advances the device position
int eng_replay(asdsl_b200_engine* e, bool decode) {
    const bool lng = e->g_decode_long != nullptr && e->host_pos >= 256;
    cudaGraphExec_t g = decode ? (lng ? e->g_decode_long : e->g_decode) : (lng ? e->g_prefill_long : e->g_prefill);
    ASDSL_CUDA(cudaGraphLaunch(g, e->stream));
    if (e->host_pos >= 0 && e->host_pos < e->cfg.max_seq_len) ++e->host_pos;
    return kOk;
}

int eng_zero_kv_from(asdsl_b200_engine* e, int from) {
    if (from < 0) from = 0;
    if (from >= e->cfg.max_seq_len) return kOk;
    const long long per_pos_codes = static_cast<long long>(e->cfg.num_kv_heads) * e->cfg.head_dim;
    const long long per_pos_scales = static_cast<long long>(e->cfg.num_kv_heads) * (e->cfg.head_dim / 64);
    asdsl::k_kv_fill<<<sm_count() * 4, 256, 0, e->stream>>>(e->kq, e->vq, e->ks, e->vs, e->cfg.num_layers,
                                                            e->kv_codes_per_layer, e->kv_scales_per_layer,
                                                            per_pos_codes * from, per_pos_scales * from);
    ASDSL_CUDA(cudaGetLastError());
    return kOk;
}

int eng_status(asdsl_b200_engine* e) {
    unsigned int* sp = device_status_ptr();
    if (!sp) return set_error(kEcuda, "cannot resolve the device status word");
    ASDSL_CUDA(cudaMemcpyAsync(&e->h_stage[3], sp, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
    ASDSL_CUDA(cudaStreamSynchronize(e->stream));
    if (e->h_stage[3] != 0) {
        // an aborted persistent step can leave its grid-barrier counter mid-count: re-arm it
        if (e->grid_bar) cudaMemsetAsync(e->grid_bar, 0, 64, e->stream);
        return set_error(kEtimeout, "engine: a kernel gave up a bounded wait (device status " +
                                        std::to_string(e->h_stage[3]) + ")");
    }
    return kOk;
}

// ---------------------------------------------------------------------------
// batched forward (UnifiedEngine::forward_batch, unified_engine.cpp:1117): the tokens of one pass
// share every weight read -- one multi-token GEMV per projection -- and give rows bit-identical
// to forward_token's:
//   * each multi-token GEMV sums a row's slices in the single-token kernel's order, with the
//     K-split of the single-token launch of the same projection (eng_single_parts);
//   * the A8 areas come from the single-token prologue code (k_quant_tokens);
//   * attention reads its own position back from the cache, which dequantizes to the values the
//     single-token head keeps in shared memory;
//   * gate/up rows are stored, then SiLU(gate) * up runs the paired epilogue's arithmetic.
// ---------------------------------------------------------------------------
__global__ void k_silu_rows(const float* __restrict__ gu, float* __restrict__ h, int I, int n) {
    const long long total = static_cast<long long>(I) * n;
    for (long long k = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; k < total;
         k += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long t = k / I;
        const long long i = k - t * I;
        h[k] = ref_silu_mul(gu[2 * t * I + i], gu[2 * t * I + I + i]);
    }
}

int eng_streams(const EngProj& p, StreamIn* in) {
    if (p.fmt == ASDSL_B200_FMT_PREQ2) preq2_streams(in, p.w0, p.w1, p.rows, p.cols);
    else q128b_streams(in, p.w0, p.w1, p.rows, p.cols);
    return p.fmt == ASDSL_B200_FMT_PREQ2 ? 32 : 128;
}

// the K-split eng_gemv's single-token launch of p uses (pair_rows > 0: the paired gate/up form)
int eng_single_parts(const EngProj& p, long long pair_rows) {
    StreamIn in[2];
    eng_streams(p, in);
    const long long M = pair_rows > 0 ? pair_rows : p.rows;
    const int nseg = pair_rows > 0 ? 2 : 1;
    const long long ub = in[0].unit_bytes + in[1].unit_bytes;
    return plan_split((M + 3) / 4, ub * nseg, nseg, FmtTraits<kFmtPreq2>::kRowsPerUnit, p.cols, LaunchOpts()).parts;
}

// T token rows through projection p (all p.rows rows, no pairing) with the K-split `parts`
template <int FMT, int PRO, int EPI>
int eng_gemv_rows_fmt(const StreamIn* in, long long nb, GemvArgs ga, int T, const LaunchOpts& o, cudaStream_t s) {
    ga.n_tokens = T;
    if (T == 1) return launch_stream_gemv<FMT, PRO, EPI, 1>(in, 2, nb, 0, ga, s, o);
    if (T >= 4)
        if (int rc = quant_tokens<PRO>(ga, T, s)) return rc;
    if (T <= 2) return launch_stream_gemv<FMT, PRO, EPI, 2>(in, 2, nb, 0, ga, s, o);
    if (T <= 4) return launch_stream_gemv<FMT, PRO, EPI, 4>(in, 2, nb, 0, ga, s, o);
    if (T <= 8) return launch_stream_gemv<FMT, PRO, EPI, 8>(in, 2, nb, 0, ga, s, o);
    return launch_stream_gemv<FMT, PRO, EPI, 16>(in, 2, nb, 0, ga, s, o);
}

// rows of one multi-token GEMV over K inputs: at most 16, and their A8 areas within a token
// scratch slot (10 for K = 8192)
int eng_rows_cap(int K) {
    const uint32_t xa = std::max(xarea_layout_bytes(K, 32, false), xarea_layout_bytes(K, 128, false));
    const int cap = static_cast<int>(kTokSlotBytes / xa);
    return cap > 16 ? 16 : (cap < 1 ? 1 : cap);
}

// T token rows through projection p with the K-split `parts`, in the fewest equal sub-passes
// that fit eng_rows_cap (row t: x + t K, y / resid + t M)
template <int PRO, int EPI>
int eng_gemv_rows(const EngProj& p, GemvArgs ga, int T, int parts, cudaStream_t s) {
    StreamIn in[2];
    ga.gs = eng_streams(p, in);
    LaunchOpts o;
    o.k_parts = parts;
    const long long nb = (static_cast<long long>(p.rows) + 3) / 4;
    const int cap = eng_rows_cap(ga.K);
    const int n_sub = (T + cap - 1) / cap;
    const int per = (T + n_sub - 1) / n_sub;
    for (int t0 = 0; t0 < T; t0 += per) {
        GemvArgs g = ga;
        const int n = std::min(per, T - t0);
        g.x = ga.x + static_cast<long long>(t0) * ga.K;
        if (ga.y) g.y = ga.y + static_cast<long long>(t0) * ga.M;
        if (ga.resid) g.resid = ga.resid + static_cast<long long>(t0) * ga.M;
        const int rc = p.fmt == ASDSL_B200_FMT_PREQ2 ? eng_gemv_rows_fmt<kFmtPreq2, PRO, EPI>(in, nb, g, n, o, s)
                                                      : eng_gemv_rows_fmt<kFmtQ128B, PRO, EPI>(in, nb, g, n, o, s);
        if (rc) return rc;
    }
    return kOk;
}

int eng_batch_alloc(asdsl_b200_engine* e) {
    if (e->batch_rows > 0) return kOk;
    const asdsl_b200_engine_config& c = e->cfg;
    const size_t B = 16;  // tokens per pass; a projection whose input is wider takes sub-passes
    const size_t qd = static_cast<size_t>(c.num_heads) * c.head_dim, kvd = static_cast<size_t>(c.num_kv_heads) * c.head_dim;
    const size_t H = c.hidden_size, I = c.intermediate_size;
    if (int rc = eng_alloc(e, &e->b_resid, 4 * B * H)) return rc;
    if (int rc = eng_alloc(e, &e->b_qkv, 4 * B * (qd + 2 * kvd))) return rc;
    if (int rc = eng_alloc(e, &e->b_att, 4 * B * qd)) return rc;
    if (int rc = eng_alloc(e, &e->b_gu, 4 * B * 2 * I)) return rc;
    if (int rc = eng_alloc(e, &e->b_h, 4 * B * I)) return rc;
    e->batch_rows = static_cast<int>(B);
    return kOk;
}

// one pass of T <= batch_rows tokens (device ids tok[0..T)) at positions start .. start + T - 1;
// logits: null, or T rows of vocab logits (all_rows) / the last token's row plus its argmax
int eng_batch_pass(asdsl_b200_engine* e, const int* tok, int T, int start, float* logits, bool all_rows) {
    const asdsl_b200_engine_config& c = e->cfg;
    cudaStream_t s = e->stream;
    const int H = c.hidden_size, I = c.intermediate_size;
    const int qkv_rows = c.num_heads * c.head_dim + 2 * c.num_kv_heads * c.head_dim;
    {
        const dim3 grid((H + 255) / 256, T);
        if (e->embed_f16) {
            const uint16_t* emb = static_cast<const uint16_t*>(e->embed);
            void* args[] = {&emb, &e->b_resid, const_cast<int**>(&tok), const_cast<int*>(&c.hidden_size)};
            if (int rc = launch_small(reinterpret_cast<const void*>(&asdsl::k_embed_rows<uint16_t>), grid, dim3(256),
                                      args, s, false))
                return rc;
        } else {
            const float* emb = static_cast<const float*>(e->embed);
            void* args[] = {&emb, &e->b_resid, const_cast<int**>(&tok), const_cast<int*>(&c.hidden_size)};
            if (int rc = launch_small(reinterpret_cast<const void*>(&asdsl::k_embed_rows<float>), grid, dim3(256),
                                      args, s, false))
                return rc;
        }
    }
    for (int l = 0; l < c.num_layers; ++l) {
        const EngLayer& L = e->layers[l];
        {
            GemvArgs ga = base_args(L.p[kProjQkv].rows, H, 32);
            ga.x = e->b_resid;
            ga.norm_w = L.rms_att;
            ga.eps = c.rms_norm_eps;
            ga.y = e->b_qkv;
            if (int rc = eng_gemv_rows<kProRmsA8, kEpiStore>(L.p[kProjQkv], ga, T, eng_single_parts(L.p[kProjQkv], 0), s))
                return rc;
        }
        {
            asdsl::AttnArgs aa;
            aa.qkv = e->b_qkv;
            aa.out = e->b_att;
            aa.kq = e->kq + l * e->kv_codes_per_layer;
            aa.vq = e->vq + l * e->kv_codes_per_layer;
            aa.ks = e->ks + l * e->kv_scales_per_layer;
            aa.vs = e->vs + l * e->kv_scales_per_layer;
            aa.cos_t = e->cos_t;
            aa.sin_t = e->sin_t;
            aa.st = nullptr;
            aa.n_heads = c.num_heads;
            aa.n_kv = c.num_kv_heads;
            aa.rot = c.rotary_dim;
            aa.max_seq = c.max_seq_len;
            int start_ = start, stride_ = qkv_rows;
            void* args[] = {&aa, &start_, &stride_};
            if (int rc = launch_small(reinterpret_cast<const void*>(&asdsl::k_kv_write_rows), dim3(c.num_kv_heads, T),
                                      dim3(asdsl::kAttnHeadDim), args, s, false))
                return rc;
            if (int rc = launch_small(reinterpret_cast<const void*>(&asdsl::k_attention_rows), dim3(c.num_heads, T),
                                      dim3(asdsl::kAttnWarps * 32), args, s, false))
                return rc;
        }
        {
            GemvArgs ga = base_args(H, L.p[kProjO].cols, 32);
            ga.x = e->b_att;
            ga.resid = e->b_resid;
            if (int rc = eng_gemv_rows<kProA8, kEpiResid>(L.p[kProjO], ga, T, eng_single_parts(L.p[kProjO], 0), s))
                return rc;
        }
        {
            GemvArgs ga = base_args(2 * I, H, 32);
            ga.x = e->b_resid;
            ga.norm_w = L.rms_ffn;
            ga.eps = c.rms_norm_eps;
            ga.y = e->b_gu;
            if (int rc = eng_gemv_rows<kProRmsA8, kEpiStore>(L.p[kProjGateUp], ga, T, eng_single_parts(L.p[kProjGateUp], I), s))
                return rc;
            const long long total = static_cast<long long>(I) * T;
            const unsigned blocks = static_cast<unsigned>(std::min<long long>((total + 255) / 256, sm_count() * 8));
            k_silu_rows<<<blocks, 256, 0, s>>>(e->b_gu, e->b_h, I, T);
            ASDSL_CUDA(cudaGetLastError());
        }
        {
            GemvArgs ga = base_args(H, I, 32);
            ga.x = e->b_h;
            ga.resid = e->b_resid;
            if (int rc = eng_gemv_rows<kProA8, kEpiResid>(L.p[kProjDown], ga, T, eng_single_parts(L.p[kProjDown], 0), s))
                return rc;
        }
    }
    if (!logits) return kOk;
    if (all_rows) {
        GemvArgs ga = base_args(c.vocab_size, H, 32);
        ga.x = e->b_resid;
        ga.norm_w = e->out_norm;
        ga.eps = c.rms_norm_eps;
        ga.y = logits;
        return eng_gemv_rows<kProRmsA8, kEpiStore>(e->lm, ga, T, eng_single_parts(e->lm, 0), s);
    }
    // the last token: the decode step's lm_head launch (logits and argmax)
    GemvArgs ga = base_args(c.vocab_size, H, 32);
    ga.x = e->b_resid + static_cast<long long>(T - 1) * H;
    ga.norm_w = e->out_norm;
    ga.eps = c.rms_norm_eps;
    ga.y = logits;
    ga.counter = reinterpret_cast<unsigned int*>(e->am_scratch);
    ga.part_val = reinterpret_cast<float*>(e->am_scratch + 256);
    ga.part_idx = reinterpret_cast<int*>(e->am_scratch + 256 + 4 * 1024);
    ga.out_val = e->am_val;
    ga.out_idx = e->am_idx;
    ga.row_base = 0;
    return eng_gemv<kProRmsA8, kEpiArgmax>(e->lm, ga, 0, s);
}

#define ENG_CHECK(e)                                                                        \
    do {                                                                                    \
        if (!(e)) return set_error(kEinval, "engine: null engine");                         \
    } while (0)
#define ENG_READY(e)                                                                        \
    do {                                                                                    \
        ENG_CHECK(e);                                                                       \
        if (!(e)->finalized) return set_error(kEinval, "engine: finalize() has not run");   \
    } while (0)

// forward_batch without the batched passes (the reference-exact mode, whose rows follow the
// reference's per-token order): n serial replays -- the decode graph where a step's logits are
// wanted, else the prefill graph -- with tokens[i] put into seq before step i; the logits of every
// step (all_logits) or of the last one.  The stream is idle on entry.
int eng_forward_serial(asdsl_b200_engine* e, const int32_t* tokens, int n, int start_pos, float* out_logits,
                       int all_logits) {
    const size_t row = 4ull * e->cfg.vocab_size;
    const bool all = out_logits && all_logits;
    if (all && e->verify_rows < n) {
        if (e->verify_logits) cudaFree(e->verify_logits);
        e->verify_logits = nullptr;
        e->verify_rows = 0;
        ASDSL_CUDA(cudaMalloc(&e->verify_logits, row * n));
        e->verify_rows = n;
    }
    ASDSL_CUDA(cudaMemcpyAsync(e->verify_tok, tokens, 4ull * n, cudaMemcpyHostToDevice, e->stream));
    if (int rc = eng_set_pos(e, start_pos, -1)) return rc;
    for (int i = 0; i < n; ++i) {
        ASDSL_CUDA(cudaMemcpyAsync(e->seq + start_pos + i, e->verify_tok + i, 4, cudaMemcpyDeviceToDevice,
                                   e->stream));
        const bool want = all || (out_logits && i == n - 1);
        if (int rc = eng_replay(e, want)) return rc;
        if (all)
            ASDSL_CUDA(cudaMemcpyAsync(reinterpret_cast<uint8_t*>(e->verify_logits) + row * i, e->logits, row,
                                       cudaMemcpyDeviceToDevice, e->stream));
    }
    if (all) ASDSL_CUDA(cudaMemcpyAsync(out_logits, e->verify_logits, row * n, cudaMemcpyDefault, e->stream));
    else if (out_logits) ASDSL_CUDA(cudaMemcpyAsync(out_logits, e->logits, row, cudaMemcpyDefault, e->stream));
    if (int rc = eng_status(e)) return rc;  // synchronizes the stream
    if (start_pos + n > e->kv_seq_len) e->kv_seq_len = start_pos + n;
    return kOk;
}

}  // namespace

extern "C" {

int asdsl_b200_engine_create(const asdsl_b200_engine_config* cfg, asdsl_b200_engine** out) {
    if (!cfg || !out) return set_error(kEinval, "engine_create: null pointer");
    *out = nullptr;
    const asdsl_b200_engine_config& c = *cfg;
    if (c.num_layers <= 0 || c.hidden_size <= 0 || c.num_heads <= 0 || c.num_kv_heads <= 0 || c.vocab_size <= 0 ||
        c.intermediate_size <= 0 || c.max_seq_len <= 0)
        return set_error(kEinval, "engine_create: dimensions must be positive");
    if (c.head_dim != 128) return set_error(kEinval, "engine_create: head_dim must be 128");
    if (c.num_heads % c.num_kv_heads) return set_error(kEinval, "engine_create: num_heads % num_kv_heads != 0");
    if (c.rotary_dim < 0 || c.rotary_dim > c.head_dim || (c.rotary_dim & 1))
        return set_error(kEinval, "engine_create: rotary_dim must be even and <= head_dim");
    if (c.weight_format != 0 || c.group_size != 32)
        return set_error(kEinval, "engine_create: only weight_format 0 with group_size 32 is supported");
    const int lm_gs = c.lm_head_group_size > 0 ? c.lm_head_group_size : c.group_size;
    if (lm_gs != 32 && lm_gs != 128) return set_error(kEinval, "engine_create: lm_head_group_size must be 32 or 128");
    if (c.hidden_size % 128 || c.intermediate_size % 128 || (c.num_heads * c.head_dim) % 128)
        return set_error(kEinval, "engine_create: hidden, intermediate and q dims must be multiples of 128");
    if (c.hidden_size > 17920 || c.intermediate_size > 17920)
        return set_error(kEinval, "engine_create: in_features exceeds 17920");
    if (sm_count() > 1024) return set_error(kEinval, "engine_create: too many SMs for the argmax scratch layout");

    auto* e = new asdsl_b200_engine();
    e->cfg = c;
    if (const char* m = std::getenv("ASDSL_B200_DECODE_KERNEL")) e->persistent = (std::string(m) == "persistent") ? 1 : 0;
    if (e->cfg.lm_head_group_size <= 0) e->cfg.lm_head_group_size = c.group_size;
    cudaGetDevice(&e->device);
    int rc = kOk;
    auto fail = [&](int code) {
        asdsl_b200_engine_destroy(e);
        return code;
    };
    if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess)
        return fail(set_error(kEcuda, "engine_create: cannot create stream"));
    const int qd = c.num_heads * c.head_dim, kvd = c.num_kv_heads * c.head_dim;
    e->layers.resize(c.num_layers);
    e->kv_codes_per_layer = static_cast<long long>(c.max_seq_len) * kvd;
    e->kv_scales_per_layer = static_cast<long long>(c.max_seq_len) * c.num_kv_heads * (c.head_dim / 64);
    if ((rc = eng_alloc(e, &e->resid, 4ull * c.hidden_size)) || (rc = eng_alloc(e, &e->qkv, 4ull * (qd + 2 * kvd))) ||
        (rc = eng_alloc(e, &e->att, 4ull * qd)) || (rc = eng_alloc(e, &e->h, 4ull * c.intermediate_size)) ||
        (rc = eng_alloc(e, &e->logits, 4ull * c.vocab_size)) ||
        (rc = eng_alloc(e, &e->kq, static_cast<size_t>(c.num_layers) * e->kv_codes_per_layer)) ||
        (rc = eng_alloc(e, &e->vq, static_cast<size_t>(c.num_layers) * e->kv_codes_per_layer)) ||
        (rc = eng_alloc(e, &e->ks, 4ull * c.num_layers * e->kv_scales_per_layer)) ||
        (rc = eng_alloc(e, &e->vs, 4ull * c.num_layers * e->kv_scales_per_layer)) ||
        (rc = eng_alloc(e, &e->st, sizeof(asdsl::DecodeState))) ||
        (rc = eng_alloc(e, &e->seq, 4ull * (c.max_seq_len + 1))) || (rc = eng_alloc(e, &e->am_val, 16)) ||
        (rc = eng_alloc(e, &e->verify_tok, 4ull * c.max_seq_len)) ||
        (rc = eng_alloc(e, &e->am_idx, 16)) ||
        (rc = eng_alloc(e, &e->am_scratch, asdsl_b200_argmax_scratch_bytes())) ||
        (rc = eng_alloc(e, &e->grid_bar, 64)) || (rc = eng_alloc(e, &e->part_val, 4ull * 1024)) ||
        (rc = eng_alloc(e, &e->part_idx, 4ull * 1024)) ||
        (rc = eng_alloc(e, &e->out_norm, 4ull * c.hidden_size)) ||
        (rc = eng_alloc(e, &e->cos_t, 4ull * c.max_seq_len * (c.rotary_dim / 2 > 0 ? c.rotary_dim / 2 : 1))) ||
        (rc = eng_alloc(e, &e->sin_t, 4ull * c.max_seq_len * (c.rotary_dim / 2 > 0 ? c.rotary_dim / 2 : 1))))
        return fail(rc);
    for (auto& L : e->layers)
        if ((rc = eng_alloc(e, &L.rms_att, 4ull * c.hidden_size)) || (rc = eng_alloc(e, &L.rms_ffn, 4ull * c.hidden_size)))
            return fail(rc);
    if ((rc = eng_alloc(e, &e->xn, 4ull * c.hidden_size)) || (rc = eng_alloc(e, &e->gu, 8ull * c.intermediate_size)))
        return fail(rc);
    e->attn_chunks = (c.max_seq_len + asdsl::kAttnChunk - 1) / asdsl::kAttnChunk;
    // ASDSL_B200_ATTN_SPLIT=0: one CTA per head over every position (the split's baseline)
    if (const char* sp = std::getenv("ASDSL_B200_ATTN_SPLIT"))
        if (sp[0] == '0') e->attn_chunks = 1;
    if (e->attn_chunks > 1) {
        if ((rc = eng_alloc(e, &e->attn_part, 4ull * c.num_heads * e->attn_chunks * asdsl::kAttnPartStride)) ||
            (rc = eng_alloc(e, &e->attn_cnt, 4ull * c.num_heads)))
            return fail(rc);
        if (cudaMemsetAsync(e->attn_cnt, 0, 4ull * c.num_heads, e->stream) != cudaSuccess)
            return fail(set_error(kEcuda, "engine_create: memset failed"));
    }
    if (cudaHostAlloc(reinterpret_cast<void**>(&e->h_stage), 16 * sizeof(int), cudaHostAllocDefault) != cudaSuccess)
        return fail(set_error(kEcuda, "engine_create: cannot allocate pinned staging"));
    if (cudaMemsetAsync(e->am_scratch, 0, asdsl_b200_argmax_scratch_bytes(), e->stream) != cudaSuccess ||
        cudaMemsetAsync(e->grid_bar, 0, 64, e->stream) != cudaSuccess ||
        cudaMemsetAsync(e->st, 0, sizeof(asdsl::DecodeState), e->stream) != cudaSuccess ||
        cudaMemsetAsync(e->seq, 0, 4ull * (c.max_seq_len + 1), e->stream) != cudaSuccess)
        return fail(set_error(kEcuda, "engine_create: memset failed"));
    if ((rc = eng_zero_kv_from(e, 0))) return fail(rc);
    if (cudaStreamSynchronize(e->stream) != cudaSuccess) return fail(set_error(kEcuda, "engine_create: sync failed"));
    *out = e;
    return kOk;
}

int asdsl_b200_engine_destroy(asdsl_b200_engine* e) {
    if (!e) return kOk;
    DeviceGuard dg(e->device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    if (e->g_decode) cudaGraphExecDestroy(e->g_decode);
    if (e->g_prefill) cudaGraphExecDestroy(e->g_prefill);
    if (e->g_decode_long) cudaGraphExecDestroy(e->g_decode_long);
    for (auto& gd : e->g_draft)
        if (gd) cudaGraphExecDestroy(gd);
    if (e->g_prefill_long) cudaGraphExecDestroy(e->g_prefill_long);
    for (void* p : e->allocs)
        if (p) cudaFree(p);
    for (auto*& p : e->d_prog)
        if (p) cudaFree(p);
    if (e->h_stage) cudaFreeHost(e->h_stage);
    if (e->verify_logits) cudaFree(e->verify_logits);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
    return kOk;
}

int asdsl_b200_engine_set_globals(asdsl_b200_engine* e, const void* token_embd, int embd_is_f16,
                                  const float* output_norm, const float* cos_table, const float* sin_table) {
    ENG_CHECK(e);
    if (!token_embd || !output_norm || !cos_table || !sin_table)
        return set_error(kEinval, "engine_set_globals: null pointer");
    if (e->finalized) return set_error(kEinval, "engine_set_globals: engine already finalized");
    DeviceGuard dg(e->device);
    const asdsl_b200_engine_config& c = e->cfg;
    const size_t esz = (embd_is_f16 ? 2ull : 4ull) * c.vocab_size * c.hidden_size;
    if (e->embed) eng_free(e, e->embed);
    e->embed = nullptr;
    if (int rc = eng_alloc(e, reinterpret_cast<uint8_t**>(&e->embed), esz)) return rc;
    e->embed_f16 = embd_is_f16 ? 1 : 0;
    const size_t half = c.rotary_dim / 2;
    ASDSL_CUDA(cudaMemcpy(e->embed, token_embd, esz, cudaMemcpyDefault));
    ASDSL_CUDA(cudaMemcpy(e->out_norm, output_norm, 4ull * c.hidden_size, cudaMemcpyDefault));
    if (half) {
        ASDSL_CUDA(cudaMemcpy(e->cos_t, cos_table, 4ull * c.max_seq_len * half, cudaMemcpyDefault));
        ASDSL_CUDA(cudaMemcpy(e->sin_t, sin_table, 4ull * c.max_seq_len * half, cudaMemcpyDefault));
    }
    return kOk;
}

int asdsl_b200_engine_set_output_proj(asdsl_b200_engine* e, const void* output_proj, int is_f16) {
    ENG_CHECK(e);
    if (!output_proj) return set_error(kEinval, "engine_set_output_proj: null pointer");
    if (e->finalized) return set_error(kEinval, "engine_set_output_proj: engine already finalized");
    DeviceGuard dg(e->device);
    const size_t sz = (is_f16 ? 2ull : 4ull) * eng_lm_rows(e) * e->cfg.hidden_size;
    if (e->out_proj) eng_free(e, e->out_proj);
    e->out_proj = nullptr;
    if (int rc = eng_alloc(e, reinterpret_cast<uint8_t**>(&e->out_proj), sz)) return rc;
    e->out_proj_f16 = is_f16 ? 1 : 0;
    ASDSL_CUDA(cudaMemcpy(e->out_proj, output_proj, sz, cudaMemcpyDefault));
    return kOk;
}

int asdsl_b200_engine_set_lm_head_preq2(asdsl_b200_engine* e, const uint8_t* meta, size_t meta_bytes,
                                        const uint8_t* quant, size_t quant_bytes) {
    ENG_CHECK(e);
    if (!meta || !quant) return set_error(kEinval, "engine_set_lm_head_preq2: null pointer");
    if (e->finalized) return set_error(kEinval, "engine_set_lm_head_preq2: engine already finalized");
    const asdsl_b200_engine_config& c = e->cfg;
    const long long ng = c.hidden_size / 32;
    const int V = eng_lm_rows(e);
    const size_t em = static_cast<size_t>(V) * ng * 4;
    const size_t eq = static_cast<size_t>((V + 3) / 4) * ng * 64;
    // as the reference constructor: blobs of the wrong size (or a g128 lm_head) are ignored
    if (c.lm_head_group_size != 32 || meta_bytes != em || quant_bytes != eq) return kOk;
    DeviceGuard dg(e->device);
    if (!e->lm.w0 || e->lm.fmt != ASDSL_B200_FMT_PREQ2) {
        if (int rc = eng_alloc(e, &e->lm.w0, em)) return rc;
        if (int rc = eng_alloc(e, &e->lm.w1, eq)) return rc;
    }
    ASDSL_CUDA(cudaMemcpy(e->lm.w0, meta, em, cudaMemcpyDefault));
    ASDSL_CUDA(cudaMemcpy(e->lm.w1, quant, eq, cudaMemcpyDefault));
    e->lm.fmt = ASDSL_B200_FMT_PREQ2;
    e->lm.rows = V;
    e->lm.cols = c.hidden_size;
    e->lm_ready = true;
    return kOk;
}

int asdsl_b200_engine_set_layer_norms(asdsl_b200_engine* e, int layer, const float* rms_att, const float* rms_ffn) {
    ENG_CHECK(e);
    if (!rms_att || !rms_ffn) return set_error(kEinval, "engine_set_layer_norms: null pointer");
    if (layer < 0 || layer >= e->cfg.num_layers) return set_error(kErange, "engine_set_layer_norms: layer out of range");
    DeviceGuard dg(e->device);
    ASDSL_CUDA(cudaMemcpy(e->layers[layer].rms_att, rms_att, 4ull * e->cfg.hidden_size, cudaMemcpyDefault));
    ASDSL_CUDA(cudaMemcpy(e->layers[layer].rms_ffn, rms_ffn, 4ull * e->cfg.hidden_size, cudaMemcpyDefault));
    return kOk;
}

int asdsl_b200_engine_set_projection(asdsl_b200_engine* e, int layer, int which, int fmt, const uint8_t* w0,
                                     size_t w0_bytes, const uint8_t* w1, size_t w1_bytes) {
    ENG_CHECK(e);
    if (e->finalized) return set_error(kEinval, "engine_set_projection: engine already finalized");
    if (layer < 0 || layer >= e->cfg.num_layers) return set_error(kErange, "engine_set_projection: layer out of range");
    if (which < 0 || which > 3) return set_error(kEinval, "engine_set_projection: projection index must be 0..3");
    if (!w0) return set_error(kEinval, "engine_set_projection: null pointer");
    DeviceGuard dg(e->device);
    int rows = 0, cols = 0;
    proj_shape(e->cfg, which, &rows, &cols);
    EngProj& p = e->layers[layer].p[which];
    if (p.w0) eng_free(e, p.w0);
    if (p.w1) eng_free(e, p.w1);
    p = EngProj();
    p.rows = rows;
    p.cols = cols;
    const long long nb = (rows + 3) / 4;
    if (fmt == ASDSL_B200_FMT_PREQ2) {
        const long long ng = cols / 32;
        const size_t em = static_cast<size_t>(rows) * ng * 4, eq = static_cast<size_t>(nb) * ng * 64;
        if (!w1) return set_error(kEinval, "engine_set_projection: null pointer");
        if (w0_bytes != em || w1_bytes != eq)
            return set_error(kEinval, "engine_set_projection: preq2 blob sizes do not match the projection shape");
        if (int rc = eng_alloc(e, &p.w0, em)) return rc;
        if (int rc = eng_alloc(e, &p.w1, eq)) return rc;
        ASDSL_CUDA(cudaMemcpy(p.w0, w0, em, cudaMemcpyDefault));
        ASDSL_CUDA(cudaMemcpy(p.w1, w1, eq, cudaMemcpyDefault));
        p.fmt = ASDSL_B200_FMT_PREQ2;
        return kOk;
    }
    if (fmt == ASDSL_B200_FMT_Q4_128) {
        const long long ng = cols / 128;
        const size_t eb = static_cast<size_t>(rows) * ng * 66;
        if (w0_bytes != eb)
            return set_error(kEinval, "engine_set_projection: Q4_128 blob size does not match the projection shape");
        uint8_t* raw = nullptr;
        if (int rc = eng_alloc(e, &raw, eb)) return rc;
        if (int rc = eng_alloc(e, &p.w0, static_cast<size_t>(nb) * ng * 256)) return rc;
        if (int rc = eng_alloc(e, &p.w1, static_cast<size_t>(nb) * ng * 8)) return rc;
        ASDSL_CUDA(cudaMemcpy(raw, w0, eb, cudaMemcpyDefault));
        int rc = asdsl_b200_relayout_q4_128(raw, p.w0, p.w1, rows, cols, e->stream);
        if (rc == kOk && cudaStreamSynchronize(e->stream) != cudaSuccess)
            rc = set_error(kEcuda, "engine_set_projection: relayout failed");
        eng_free(e, raw);
        if (rc) return rc;
        p.fmt = ASDSL_B200_FMT_Q4_128_BANDED;
        return kOk;
    }
    return set_error(kEinval, "engine_set_projection: fmt must be PREQ2 or Q4_128");
}

int asdsl_b200_engine_finalize(asdsl_b200_engine* e) {
    ENG_CHECK(e);
    if (e->finalized) return kOk;
    DeviceGuard dg(e->device);
    const asdsl_b200_engine_config& c = e->cfg;
    if (!e->embed) return set_error(kEinval, "engine_finalize: set_globals() has not run");
    for (int l = 0; l < c.num_layers; ++l)
        for (int w = 0; w < 4; ++w)
            if (e->layers[l].p[w].fmt < 0)
                return set_error(kEinval, "engine_finalize: layer " + std::to_string(l) + " projection " +
                                              std::to_string(w) + " has no weights");
    if (!e->lm_ready) {
        if (!e->out_proj) return set_error(kEinval, "engine_finalize: no lm_head source (output_proj or preq2 blobs)");
        const int V = eng_lm_rows(e);
        const long long nb = (V + 3) / 4;
        const unsigned blocks = static_cast<unsigned>(sm_count() * 8);
        if (c.lm_head_group_size == 32) {
            const long long ng = c.hidden_size / 32;
            if (int rc = eng_alloc(e, &e->lm.w0, static_cast<size_t>(V) * ng * 4)) return rc;
            if (int rc = eng_alloc(e, &e->lm.w1, static_cast<size_t>(nb) * ng * 64)) return rc;
            ASDSL_CUDA(cudaMemsetAsync(e->lm.w1, 0, static_cast<size_t>(nb) * ng * 64, e->stream));
            if (e->out_proj_f16)
                asdsl::k_lmhead_quant_preq2<uint16_t><<<blocks, 256, 0, e->stream>>>(
                    static_cast<const uint16_t*>(e->out_proj), reinterpret_cast<uint32_t*>(e->lm.w0),
                    reinterpret_cast<uint4*>(e->lm.w1), V, c.hidden_size);
            else
                asdsl::k_lmhead_quant_preq2<float><<<blocks, 256, 0, e->stream>>>(
                    static_cast<const float*>(e->out_proj), reinterpret_cast<uint32_t*>(e->lm.w0),
                    reinterpret_cast<uint4*>(e->lm.w1), V, c.hidden_size);
            e->lm.fmt = ASDSL_B200_FMT_PREQ2;
        } else {
            const long long ng = c.hidden_size / 128;
            if (int rc = eng_alloc(e, &e->lm.w0, static_cast<size_t>(nb) * ng * 256)) return rc;
            if (int rc = eng_alloc(e, &e->lm.w1, static_cast<size_t>(nb) * ng * 8)) return rc;
            ASDSL_CUDA(cudaMemsetAsync(e->lm.w0, 0, static_cast<size_t>(nb) * ng * 256, e->stream));
            ASDSL_CUDA(cudaMemsetAsync(e->lm.w1, 0, static_cast<size_t>(nb) * ng * 8, e->stream));
            if (e->out_proj_f16)
                asdsl::k_lmhead_quant_q128b<uint16_t><<<blocks, 256, 0, e->stream>>>(
                    static_cast<const uint16_t*>(e->out_proj), reinterpret_cast<uint4*>(e->lm.w0),
                    reinterpret_cast<uint16_t*>(e->lm.w1), V, c.hidden_size);
            else
                asdsl::k_lmhead_quant_q128b<float><<<blocks, 256, 0, e->stream>>>(
                    static_cast<const float*>(e->out_proj), reinterpret_cast<uint4*>(e->lm.w0),
                    reinterpret_cast<uint16_t*>(e->lm.w1), V, c.hidden_size);
            e->lm.fmt = ASDSL_B200_FMT_Q4_128_BANDED;
        }
        ASDSL_CUDA(cudaGetLastError());
        e->lm.rows = V;
        e->lm.cols = c.hidden_size;
        ASDSL_CUDA(cudaStreamSynchronize(e->stream));
        e->lm_ready = true;
    }
    if (e->vx && (e->exact || e->persistent))
        return set_error(kEinval, "engine_finalize: a sharded engine runs the fast per-op chain");
    if (e->exact) {
        // the reference-exact mode covers the C0 path: preq2 gs 32 everywhere (lm_head included)
        for (int l = 0; l < c.num_layers; ++l)
            for (int w = 0; w < 4; ++w)
                if (e->layers[l].p[w].fmt != ASDSL_B200_FMT_PREQ2)
                    return set_error(kEinval, "engine_finalize: the reference-exact mode needs preq2 (gs 32) projections");
        if (e->lm.fmt != ASDSL_B200_FMT_PREQ2)
            return set_error(kEinval, "engine_finalize: the reference-exact mode needs a gs 32 (preq2) lm_head");
        if (c.head_dim != asdsl::kAttnHeadDim || c.max_seq_len > asdsl::kAttnXMaxSeq || c.hidden_size % 8 ||
            c.intermediate_size % 4)
            return set_error(kEinval, "engine_finalize: the reference-exact mode needs head_dim 128, max_seq_len <= " +
                                          std::to_string(asdsl::kAttnXMaxSeq) + " and hidden_size % 8 == 0");
        if (e->persistent) return set_error(kEinval, "engine_finalize: the reference-exact mode runs the per-op chain");
        if (int rc = exact_tabs_device(&e->ex)) return rc;
        ASDSL_CUDA(cudaFuncSetAttribute(reinterpret_cast<const void*>(&asdsl::k_attention_exact),
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(asdsl::attn_x_layout(c.max_seq_len).total)));
        // every matrix into the exact layout (group-interleaved units; pure byte moves, once)
        auto relayout = [&](EngProj& p, long long pair_rows) -> int {
            const long long ng = p.cols / 32;
            const long long m_seg = pair_rows > 0 ? pair_rows : p.rows;
            const int L = asdsl::exact_lpt_for(m_seg, pair_rows > 0);
            const long long units = ((p.rows + 3) / 4 + L - 1) / L;
            uint8_t *mx = nullptr, *qx = nullptr;
            if (int rc = eng_alloc(e, &mx, static_cast<size_t>(units * ng * 16 * L))) return rc;
            if (int rc = eng_alloc(e, &qx, static_cast<size_t>(units * ng * 64 * L))) return rc;
            const long long items = units * ng * 4 * L;
            const unsigned blocks = static_cast<unsigned>(std::min<long long>((items + 255) / 256, sm_count() * 32ll));
            asdsl::k_relayout_exact<<<blocks, 256, 0, e->stream>>>(p.w0, p.w1, mx, qx, p.rows, static_cast<int>(ng), L,
                                                                   units);
            ASDSL_CUDA(cudaGetLastError());
            ASDSL_CUDA(cudaStreamSynchronize(e->stream));
            eng_free(e, p.w0);
            eng_free(e, p.w1);
            p.w0 = mx;
            p.w1 = qx;
            p.xlpt = L;
            return kOk;
        };
        for (int l = 0; l < c.num_layers; ++l) {
            EngLayer& L = e->layers[l];
            if (int rc = relayout(L.p[kProjQkv], 0)) return rc;
            if (int rc = relayout(L.p[kProjO], 0)) return rc;
            if (int rc = relayout(L.p[kProjGateUp], c.intermediate_size)) return rc;
            if (int rc = relayout(L.p[kProjDown], 0)) return rc;
        }
        if (int rc = relayout(e->lm, 0)) return rc;
#ifdef ASDSL_HOST_X86
        e->inv_sqrt_d = asdsl::host_nr_rsqrt(static_cast<float>(c.head_dim));
#endif
    }
    // the lm_head source is no longer needed (the reference drops it too)
    if (e->out_proj) {
        eng_free(e, e->out_proj);
        e->out_proj = nullptr;
    }
    if (e->persistent) {
        if (int rc = eng_build_program(e, true)) return rc;
        if (int rc = eng_build_program(e, false)) return rc;
    }
    // one eager step of each kind (kernel attributes, module loading), then capture
    if (int rc = eng_set_pos(e, 0, 0)) return rc;
    if (int rc = eng_enqueue_step(e, true)) return rc;
    if (int rc = eng_set_pos(e, 0, 0)) return rc;
    if (int rc = eng_enqueue_step(e, false)) return rc;
    ASDSL_CUDA(cudaStreamSynchronize(e->stream));
    if (int rc = eng_status(e)) return rc;
    if (int rc = eng_capture(e, true, &e->g_decode)) return rc;
    if (int rc = eng_capture(e, false, &e->g_prefill)) return rc;
    if (!e->persistent && c.max_seq_len > 256) {
        // the long-cache step graphs (one eager step of each kind first, as above)
        if (e->exact) {
            const int mt = (c.max_seq_len + asdsl::kAttnXTile - 1) / asdsl::kAttnXTile;
            asdsl::AttnXSplit& x = e->xsplit;
            if (int rc = eng_alloc(e, &x.s, 4ull * c.num_heads * c.max_seq_len)) return rc;
            if (int rc = eng_alloc(e, &x.tmax, 4ull * c.num_heads * mt)) return rc;
            if (int rc = eng_alloc(e, &x.tres, 4ull * c.num_heads * mt * asdsl::kAttnXResStride)) return rc;
            if (int rc = eng_alloc(e, &x.cnt, 4ull * c.num_heads)) return rc;
            ASDSL_CUDA(cudaMemsetAsync(x.cnt, 0, 4ull * c.num_heads, e->stream));
        }
        e->capture_long = true;
        int rc = eng_set_pos(e, 0, 0);
        if (!rc) rc = eng_enqueue_step(e, true);
        if (!rc) rc = eng_set_pos(e, 0, 0);
        if (!rc) rc = eng_enqueue_step(e, false);
        if (!rc && cudaStreamSynchronize(e->stream) != cudaSuccess) rc = set_error(kEcuda, "engine_finalize: step failed");
        if (!rc) rc = eng_status(e);
        if (!rc) rc = eng_capture(e, true, &e->g_decode_long);
        if (!rc) rc = eng_capture(e, false, &e->g_prefill_long);
        e->capture_long = false;
        if (rc) return rc;
    }
    if (int rc = eng_zero_kv_from(e, 0)) return rc;
    ASDSL_CUDA(cudaStreamSynchronize(e->stream));
    e->kv_seq_len = 0;
    e->finalized = true;
    return kOk;
}

int asdsl_b200_engine_forward_token(asdsl_b200_engine* e, int token, int pos, float* logits, int32_t* argmax) {
    ENG_READY(e);
    if (token < 0 || token >= e->cfg.vocab_size)
        return set_error(kErange, "forward_token: token_id out of vocab range");
    if (pos < 0 || pos >= e->cfg.max_seq_len) return set_error(kErange, "forward_token: pos out of kv-cache range");
    if (logits && e->vx)
        return set_error(kEinval, "forward_token: a sharded engine returns the argmax (its logits are split over ranks)");
    DeviceGuard dg(e->device);
    if (int rc = eng_set_pos(e, pos, token)) return rc;
    const bool lm = logits || argmax;
    if (int rc = eng_replay(e, lm)) return rc;
    if (logits)
        ASDSL_CUDA(cudaMemcpyAsync(logits, e->logits, 4ull * e->cfg.vocab_size, cudaMemcpyDefault, e->stream));
    if (argmax) ASDSL_CUDA(cudaMemcpyAsync(&e->h_stage[2], e->am_idx, 4, cudaMemcpyDeviceToHost, e->stream));
    if (int rc = eng_status(e)) return rc;  // synchronizes the stream
    if (argmax) *argmax = e->h_stage[2];
    if (pos + 1 > e->kv_seq_len) e->kv_seq_len = pos + 1;
    return kOk;
}

// forward_verify_serial (unified_engine.cpp:1767-1772): forward_token(tokens[i], start_pos + i) for
// i < n, logits of every step.  All n steps run back to back on the engine stream: before step
// i + 1 the token the decode step wrote into seq[start_pos + i + 1] (its argmax) is replaced by
// tokens[i + 1], and each step's logits go to row i of a device block copied out once.
int asdsl_b200_engine_forward_verify(asdsl_b200_engine* e, const int32_t* tokens, int n, int start_pos,
                                     float* out_logits) {
    ENG_READY(e);
    if (e->vx) return set_error(kEinval, "forward_verify: not available on a sharded engine");
    if (n <= 0) return kOk;
    if (!tokens || !out_logits) return set_error(kEinval, "forward_verify: null pointer");
    const asdsl_b200_engine_config& c = e->cfg;
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= c.vocab_size)
            return set_error(kErange, "forward_token: token_id out of vocab range");
    if (start_pos < 0 || start_pos >= c.max_seq_len || n > c.max_seq_len - start_pos)
        return set_error(kErange, "forward_token: pos out of kv-cache range");
    DeviceGuard dg(e->device);
    ASDSL_CUDA(cudaStreamSynchronize(e->stream));
    const size_t row = 4ull * c.vocab_size;
    if (e->verify_rows < n) {
        if (e->verify_logits) cudaFree(e->verify_logits);
        e->verify_logits = nullptr;
        e->verify_rows = 0;
        ASDSL_CUDA(cudaMalloc(&e->verify_logits, row * n));
        e->verify_rows = n;
    }
    ASDSL_CUDA(cudaMemcpyAsync(e->verify_tok, tokens, 4ull * n, cudaMemcpyHostToDevice, e->stream));
    if (int rc = eng_set_pos(e, start_pos, tokens[0])) return rc;
    for (int i = 0; i < n; ++i) {
        if (i > 0)
            ASDSL_CUDA(cudaMemcpyAsync(e->seq + start_pos + i, e->verify_tok + i, 4, cudaMemcpyDeviceToDevice,
                                       e->stream));
        if (int rc = eng_replay(e, true)) return rc;
        ASDSL_CUDA(cudaMemcpyAsync(reinterpret_cast<uint8_t*>(e->verify_logits) + row * i, e->logits, row,
                                   cudaMemcpyDeviceToDevice, e->stream));
    }
    ASDSL_CUDA(cudaMemcpyAsync(out_logits, e->verify_logits, row * n, cudaMemcpyDefault, e->stream));
    if (int rc = eng_status(e)) return rc;  // synchronizes the stream
    if (start_pos + n > e->kv_seq_len) e->kv_seq_len = start_pos + n;
    return kOk;
}

// UnifiedEngine::forward_batch (unified_engine.cpp:1117): tokens[i] at position start_pos + i
// for i < n, passes of up to batch_rows tokens through the multi-token GEMVs.  out_logits: null,
// the last token's logits (all_logits = 0), or n rows (all_logits != 0, as forward_verify_batch's
// forward_batch(..., true) call).  Rows and KV cache are bit-identical to n forward_token calls
// of the per-op decode chain.
int asdsl_b200_engine_forward_batch(asdsl_b200_engine* e, const int32_t* tokens, int n, int start_pos,
                                    float* out_logits, int all_logits) {
    ENG_READY(e);
    if (e->vx) return set_error(kEinval, "forward_batch: not available on a sharded engine");
    if (n <= 0) return kOk;
    if (!tokens) return set_error(kEinval, "forward_batch: null pointer");
    const asdsl_b200_engine_config& c = e->cfg;
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= c.vocab_size)
            return set_error(kErange, "forward_token: token_id out of vocab range");
    if (start_pos < 0 || start_pos >= c.max_seq_len || n > c.max_seq_len - start_pos)
        return set_error(kErange, "forward_token: pos out of kv-cache range");
    DeviceGuard dg(e->device);
    ASDSL_CUDA(cudaStreamSynchronize(e->stream));
    if (e->exact) return eng_forward_serial(e, tokens, n, start_pos, out_logits, all_logits);
    if (int rc = eng_batch_alloc(e)) return rc;
    const size_t row = 4ull * c.vocab_size;
    const bool all = out_logits && all_logits;
    if (all && e->verify_rows < n) {
        if (e->verify_logits) cudaFree(e->verify_logits);
        e->verify_logits = nullptr;
        e->verify_rows = 0;
        ASDSL_CUDA(cudaMalloc(&e->verify_logits, row * n));
        e->verify_rows = n;
    }
    ASDSL_CUDA(cudaMemcpyAsync(e->verify_tok, tokens, 4ull * n, cudaMemcpyHostToDevice, e->stream));
    const int B = e->batch_rows;
    for (int t0 = 0; t0 < n; t0 += B) {
        const int T = std::min(B, n - t0);
        float* lg = nullptr;
        if (all) lg = e->verify_logits + static_cast<size_t>(t0) * c.vocab_size;
        else if (out_logits && t0 + T == n) lg = e->logits;
        if (int rc = eng_batch_pass(e, e->verify_tok + t0, T, start_pos + t0, lg, all)) return rc;
    }
    if (all) ASDSL_CUDA(cudaMemcpyAsync(out_logits, e->verify_logits, row * n, cudaMemcpyDefault, e->stream));
    else if (out_logits) ASDSL_CUDA(cudaMemcpyAsync(out_logits, e->logits, row, cudaMemcpyDefault, e->stream));
    if (int rc = eng_status(e)) return rc;  // synchronizes the stream
    if (start_pos + n > e->kv_seq_len) e->kv_seq_len = start_pos + n;
    return kOk;
}

int asdsl_b200_engine_generate(asdsl_b200_engine* e, const int32_t* prompt, int n_prompt, int max_tokens,
                               const int32_t* stops, int n_stops, int32_t* out, int out_cap, int* n_out) {
    ENG_READY(e);
    if (!prompt || !out || !n_out || (n_stops > 0 && !stops)) return set_error(kEinval, "generate: null pointer");
    if (n_prompt <= 0) return set_error(kEinval, "generate: the prompt must hold at least one token");
    if (max_tokens < 0) max_tokens = 0;
    const asdsl_b200_engine_config& c = e->cfg;
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= c.vocab_size)
            return set_error(kErange, "forward_token: token_id out of vocab range");
    if (n_prompt > c.max_seq_len) return set_error(kErange, "forward_token: pos out of kv-cache range");
    // tokens t_0..t_{T-1}; t_j needs the forward of position n + j - 1 (< max_seq)
    const int room = c.max_seq_len - n_prompt;  // forwards of generated tokens that fit
    const int producible = max_tokens <= room ? max_tokens : room + 1;
    if (out_cap < n_prompt + producible) return set_error(kEinval, "generate: output buffer too small");
    DeviceGuard dg(e->device);
    ASDSL_CUDA(cudaStreamSynchronize(e->stream));
    ASDSL_CUDA(cudaMemcpyAsync(e->seq, prompt, 4ull * n_prompt, cudaMemcpyHostToDevice, e->stream));
    // prompt tokens before the last one: batched passes (bit-identical to the per-op chain's
    // prefill graph); the persistent-kernel and reference-exact modes replay their prefill graph
    const int n_pre = n_prompt - 1;
    if (n_pre > 0 && !e->persistent && !e->exact && !e->vx) {
        if (int rc = eng_batch_alloc(e)) return rc;
        for (int t0 = 0; t0 < n_pre; t0 += e->batch_rows) {
            const int T = std::min(e->batch_rows, n_pre - t0);
            if (int rc = eng_batch_pass(e, e->seq + t0, T, t0, nullptr, false)) return rc;
        }
        if (int rc = eng_set_pos(e, n_pre, -1)) return rc;
    } else {
        if (int rc = eng_set_pos(e, 0, -1)) return rc;
        for (int i = 0; i + 1 < n_prompt; ++i)
            if (int rc = eng_replay(e, false)) return rc;
    }
    // the last prompt token's forward is the first decode step; without one it is a prefill step
    if (producible == 0)
        if (int rc = eng_replay(e, false)) return rc;
    int produced = 0, stop_at = -1;
    const int chunk = n_stops > 0 ? 16 : (producible > 0 ? producible : 1);
    while (produced < producible && stop_at < 0) {
        const int n = std::min(chunk, producible - produced);
        for (int i = 0; i < n; ++i)
            if (int rc = eng_replay(e, true)) return rc;
        ASDSL_CUDA(cudaMemcpyAsync(out + n_prompt + produced, e->seq + n_prompt + produced, 4ull * n,
                                   cudaMemcpyDeviceToHost, e->stream));
        if (int rc = eng_status(e)) return rc;
        for (int i = 0; i < n && n_stops > 0; ++i) {
            const int t = out[n_prompt + produced + i];
            for (int s = 0; s < n_stops; ++s)
                if (stops[s] == t) {
                    stop_at = produced + i;
                    break;
                }
            if (stop_at >= 0) break;
        }
        produced += n;
    }
    for (int i = 0; i < n_prompt; ++i) out[i] = prompt[i];
    if (stop_at >= 0) {
        // the reference forwards t_0..t_{s-1}: keep KV below n + s
        const int kv = n_prompt + stop_at;
        if (int rc = eng_zero_kv_from(e, kv)) return rc;
        ASDSL_CUDA(cudaStreamSynchronize(e->stream));
        e->kv_seq_len = std::max(e->kv_seq_len, kv);
        *n_out = n_prompt + stop_at + 1;
        return kOk;
    }
    if (max_tokens > room) {
        // the reference's forward of t_room at position max_seq throws
        e->kv_seq_len = c.max_seq_len;
        *n_out = n_prompt + produced;
        return set_error(kErange, "forward_token: pos out of kv-cache range");
    }
    if (max_tokens > 0) {
        // forward of the last token (KV only), as the reference's loop does
        if (int rc = eng_replay(e, false)) return rc;
    }
    if (int rc = eng_status(e)) return rc;
    e->kv_seq_len = std::max(e->kv_seq_len, n_prompt + max_tokens);
    *n_out = n_prompt + produced;
    return kOk;
}

int asdsl_b200_engine_profile_step(asdsl_b200_engine* e, int decode, unsigned long long* host_trace, int max_ops,
                                   int* n_ops) {
    ENG_READY(e);
    if (!host_trace || !n_ops) return set_error(kEinval, "engine_profile_step: null pointer");
    if (!e->persistent) return set_error(kEinval, "engine_profile_step: needs the persistent decode kernel");
    DeviceGuard dg(e->device);
    asdsl::StepArgs A = e->prog_args[decode ? 1 : 0];
    if (max_ops < A.n_ops) return set_error(kEinval, "engine_profile_step: trace buffer too small");
    unsigned long long* d = nullptr;
    ASDSL_CUDA(cudaMalloc(reinterpret_cast<void**>(&d), 3ull * A.n_ops * sizeof(unsigned long long)));
    std::vector<unsigned long long> init(3ull * A.n_ops, 0ull);
    for (int i = 0; i < A.n_ops; ++i) init[3 * i] = ~0ull;
    cudaError_t ce = cudaMemcpy(d, init.data(), init.size() * sizeof(unsigned long long), cudaMemcpyHostToDevice);
    A.trace = d;
    int rc = kOk;
    if (ce != cudaSuccess) {
        rc = set_error(kEcuda, "engine_profile_step: copy failed");
    } else {
        // one eager step with the trace on, at the current position
        e->prog_args[decode ? 1 : 0].trace = d;
        rc = eng_launch_program(e, decode != 0);
        e->prog_args[decode ? 1 : 0].trace = nullptr;
        if (rc == kOk && cudaStreamSynchronize(e->stream) != cudaSuccess) rc = set_error(kEcuda, "engine_profile_step: step failed");
        if (rc == kOk && cudaMemcpy(host_trace, d, init.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost) != cudaSuccess)
            rc = set_error(kEcuda, "engine_profile_step: copy back failed");
    }
    cudaFree(d);
    *n_ops = A.n_ops;
    if (rc == kOk) rc = eng_status(e);
    return rc;
}

int asdsl_b200_engine_set_shard(asdsl_b200_engine* e, asdsl_b200_vxchg* vx, asdsl_b200_xchg* xg, int lm_rows,
                                int lm_row_base) {
    ENG_CHECK(e);
    if (e->finalized) return set_error(kEinval, "engine_set_shard: engine already finalized");
    if (e->lm_ready || e->out_proj) return set_error(kEinval, "engine_set_shard: call before the lm_head is set");
    if (!vx || !xg || !vx->open || !xg->open) return set_error(kEinval, "engine_set_shard: exchanges not opened");
    if (vx->world != xg->world || vx->rank != xg->rank)
        return set_error(kEinval, "engine_set_shard: the two exchanges disagree on rank / world");
    if (vx->device != e->device || xg->device != e->device)
        return set_error(kEinval, "engine_set_shard: the exchanges live on another device");
    const asdsl_b200_engine_config& c = e->cfg;
    if (vx->n_max < c.hidden_size) return set_error(kEinval, "engine_set_shard: vector exchange shorter than hidden_size");
    if (lm_rows <= 0 || lm_row_base < 0 || static_cast<long long>(lm_row_base) + lm_rows > c.vocab_size)
        return set_error(kErange, "engine_set_shard: lm_head rows outside the vocabulary");
    if (static_cast<long long>(lm_row_base) + lm_rows > (1ll << 24))
        return set_error(kErange, "engine_set_shard: global row indices must stay below 2^24");
    DeviceGuard dg(e->device);
    if (!e->part)
        if (int rc = eng_alloc(e, &e->part, 4ull * c.hidden_size)) return rc;
    e->vx = vx;
    e->xg = xg;
    e->lm_rows = lm_rows;
    e->lm_row_base = lm_row_base;
    return kOk;
}

// drop the captured draft-step graphs (the mask or the draft bank changed)
static void eng_drop_draft_graphs(asdsl_b200_engine* e) {
    for (auto& gd : e->g_draft) {
        if (gd) cudaGraphExecDestroy(gd);
        gd = nullptr;
    }
}

int asdsl_b200_engine_set_skip_mask(asdsl_b200_engine* e, const uint8_t* mask, int n) {
    ENG_CHECK(e);
    if (n > 0 && !mask) return set_error(kEinval, "engine_set_skip_mask: null pointer");
    DeviceGuard dg(e->device);
    ASDSL_CUDA(cudaStreamSynchronize(e->stream));
    const int lim = n < 64 ? (n > 0 ? n : 0) : 64;
    for (int i = 0; i < 64; ++i) e->skip[i] = i < lim ? mask[i] != 0 : false;
    eng_drop_draft_graphs(e);
    return kOk;
}

int asdsl_b200_engine_clear_skip_mask(asdsl_b200_engine* e) {
    ENG_CHECK(e);
    return asdsl_b200_engine_set_skip_mask(e, nullptr, 0);
}

int asdsl_b200_engine_set_projection_q2(asdsl_b200_engine* e, int layer, int which, const uint8_t* w_packed,
                                        size_t w_bytes, const float* scales, const float* biases, size_t n_groups) {
    ENG_CHECK(e);
    if (layer < 0 || layer >= e->cfg.num_layers) return set_error(kErange, "engine_set_projection_q2: layer out of range");
    if (which < 0 || which > 3) return set_error(kEinval, "engine_set_projection_q2: projection index must be 0..3");
    if (!w_packed || !scales || !biases) return set_error(kEinval, "engine_set_projection_q2: null pointer");
    int rows = 0, cols = 0;
    proj_shape(e->cfg, which, &rows, &cols);
    if (w_bytes != static_cast<size_t>(rows) * cols / 4 || n_groups != static_cast<size_t>(rows) * (cols / 32))
        return set_error(kEinval, "engine_set_projection_q2: sizes do not match the projection (packed 2-bit, gs 32)");
    DeviceGuard dg(e->device);
    ASDSL_CUDA(cudaStreamSynchronize(e->stream));
    Q2Proj& q = e->layers[layer].q2[which];
    if (!q.w) {
        if (int rc = eng_alloc(e, &q.w, w_bytes)) return rc;
        if (int rc = eng_alloc(e, &q.s, 4 * n_groups)) return rc;
        if (int rc = eng_alloc(e, &q.b, 4 * n_groups)) return rc;
    }
    ASDSL_CUDA(cudaMemcpy(q.w, w_packed, w_bytes, cudaMemcpyDefault));
    ASDSL_CUDA(cudaMemcpy(q.s, scales, 4 * n_groups, cudaMemcpyDefault));
    ASDSL_CUDA(cudaMemcpy(q.b, biases, 4 * n_groups, cudaMemcpyDefault));
    const size_t smem = 4ull * (cols + cols / 32);
    if (smem > 48 * 1024)
        ASDSL_CUDA(cudaFuncSetAttribute(reinterpret_cast<const void*>(&asdsl::k_gemv_q2<true>),
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    eng_drop_draft_graphs(e);
    return kOk;
}

int asdsl_b200_engine_forward_token_draft(asdsl_b200_engine* e, int token, int pos, float* logits, int32_t* argmax,
                                          int use_q2) {
    ENG_READY(e);
    if (e->exact || e->persistent || e->vx)
        return set_error(kEinval, "forward_token_draft: draft steps run in the fast per-op chain of one GPU");
    if (token < 0 || token >= e->cfg.vocab_size)
        return set_error(kErange, "forward_token: token_id out of vocab range");
    if (pos < 0 || pos >= e->cfg.max_seq_len) return set_error(kErange, "forward_token: pos out of kv-cache range");
    DeviceGuard dg(e->device);
    if (int rc = eng_set_pos(e, pos, token)) return rc;
    const bool lng = e->g_decode_long != nullptr && pos >= 256;
    const int key = (use_q2 ? 2 : 0) + (lng ? 1 : 0);
    if (!e->g_draft[key]) {
        // first use of this kind: the step runs as enqueued, then its graph is captured for later ones
        e->draft_skip = true;
        e->draft_q2 = use_q2 != 0;
        e->capture_long = lng;
        int rc = eng_enqueue_step(e, true);
        if (!rc) rc = eng_capture(e, true, &e->g_draft[key]);
        e->draft_skip = e->draft_q2 = e->capture_long = false;
        if (rc) return rc;
    } else {
        ASDSL_CUDA(cudaGraphLaunch(e->g_draft[key], e->stream));
    }
    if (e->host_pos >= 0 && e->host_pos < e->cfg.max_seq_len) ++e->host_pos;
    if (logits)
        ASDSL_CUDA(cudaMemcpyAsync(logits, e->logits, 4ull * e->cfg.vocab_size, cudaMemcpyDefault, e->stream));
    if (argmax) ASDSL_CUDA(cudaMemcpyAsync(&e->h_stage[2], e->am_idx, 4, cudaMemcpyDeviceToHost, e->stream));
    if (int rc = eng_status(e)) return rc;  // synchronizes the stream
    if (argmax) *argmax = e->h_stage[2];
    if (pos + 1 > e->kv_seq_len) e->kv_seq_len = pos + 1;
    return kOk;
}

int asdsl_b200_engine_set_numerics(asdsl_b200_engine* e, int mode) {
    ENG_CHECK(e);
    if (e->finalized) return set_error(kEinval, "engine_set_numerics: engine already finalized");
    if (mode != ASDSL_B200_NUMERICS_FAST && mode != ASDSL_B200_NUMERICS_REFERENCE_EXACT)
        return set_error(kEinval, "engine_set_numerics: unknown mode");
    e->exact = mode == ASDSL_B200_NUMERICS_REFERENCE_EXACT ? 1 : 0;
    return kOk;
}

int asdsl_b200_engine_set_persistent(asdsl_b200_engine* e, int persistent) {
    ENG_CHECK(e);
    if (e->finalized) return set_error(kEinval, "engine_set_persistent: engine already finalized");
    e->persistent = persistent ? 1 : 0;
    return kOk;
}

int asdsl_b200_engine_replay(asdsl_b200_engine* e, int decode, int n) {
    ENG_READY(e);
    if (n < 0) return set_error(kEinval, "engine_replay: n must be >= 0");
    DeviceGuard dg(e->device);
    for (int i = 0; i < n; ++i)
        if (int rc = eng_replay(e, decode != 0)) return rc;
    return kOk;
}

int asdsl_b200_engine_set_position(asdsl_b200_engine* e, int pos, int token) {
    ENG_READY(e);
    if (pos < 0 || pos >= e->cfg.max_seq_len) return set_error(kErange, "engine_set_position: pos out of range");
    if (token >= e->cfg.vocab_size) return set_error(kErange, "engine_set_position: token out of range");
    DeviceGuard dg(e->device);
    return eng_set_pos(e, pos, token);
}

int asdsl_b200_engine_stream(asdsl_b200_engine* e, void** stream) {
    ENG_CHECK(e);
    if (!stream) return set_error(kEinval, "engine_stream: null pointer");
    *stream = e->stream;
    return kOk;
}

int asdsl_b200_engine_reset_session(asdsl_b200_engine* e) {
    ENG_CHECK(e);
    DeviceGuard dg(e->device);
    if (int rc = eng_zero_kv_from(e, 0)) return rc;
    ASDSL_CUDA(cudaStreamSynchronize(e->stream));
    e->kv_seq_len = 0;
    e->snapshots.clear();
    // as the reference's reset_session (unified_engine.cpp:1325-1337): the skip mask is cleared
    return asdsl_b200_engine_clear_skip_mask(e);
}

int asdsl_b200_engine_get_kv_seq_len(asdsl_b200_engine* e, int* out) {
    ENG_CHECK(e);
    if (!out) return set_error(kEinval, "get_kv_seq_len: null pointer");
    *out = e->kv_seq_len;
    return kOk;
}

int asdsl_b200_engine_truncate_kv(asdsl_b200_engine* e, int new_len) {
    ENG_CHECK(e);
    if (new_len < 0) new_len = 0;
    if (new_len > e->cfg.max_seq_len) new_len = e->cfg.max_seq_len;
    DeviceGuard dg(e->device);
    if (int rc = eng_zero_kv_from(e, new_len)) return rc;
    ASDSL_CUDA(cudaStreamSynchronize(e->stream));
    e->kv_seq_len = new_len;
    return kOk;
}

int asdsl_b200_engine_snapshot_kv(asdsl_b200_engine* e) {
    ENG_CHECK(e);
    e->snapshots.push_back(e->kv_seq_len);
    return kOk;
}

int asdsl_b200_engine_restore_kv(asdsl_b200_engine* e) {
    ENG_CHECK(e);
    if (e->snapshots.empty()) return kOk;
    const int len = e->snapshots.back();
    e->snapshots.pop_back();
    return asdsl_b200_engine_truncate_kv(e, len);
}

int asdsl_b200_engine_export_lm_head(asdsl_b200_engine* e, int* fmt, uint8_t* w0, size_t w0_bytes, uint8_t* w1,
                                     size_t w1_bytes) {
    ENG_READY(e);
    if (!fmt) return set_error(kEinval, "export_lm_head: null pointer");
    if (e->lm.xlpt)
        return set_error(kEinval, "export_lm_head: the reference-exact mode keeps the lm_head in its own layout");
    if (e->vx) return set_error(kEinval, "export_lm_head: a sharded engine holds only its rows of the lm_head");
    const asdsl_b200_engine_config& c = e->cfg;
    const long long nb = (c.vocab_size + 3) / 4;
    size_t b0, b1;
    if (e->lm.fmt == ASDSL_B200_FMT_PREQ2) {
        b0 = static_cast<size_t>(c.vocab_size) * (c.hidden_size / 32) * 4;
        b1 = static_cast<size_t>(nb) * (c.hidden_size / 32) * 64;
    } else {
        b0 = static_cast<size_t>(nb) * (c.hidden_size / 128) * 256;
        b1 = static_cast<size_t>(nb) * (c.hidden_size / 128) * 8;
    }
    *fmt = e->lm.fmt;
    if (!w0 && !w1) return kOk;  // size query
    if (!w0 || !w1 || w0_bytes < b0 || w1_bytes < b1) return set_error(kEinval, "export_lm_head: buffers too small");
    DeviceGuard dg(e->device);
    ASDSL_CUDA(cudaMemcpy(w0, e->lm.w0, b0, cudaMemcpyDefault));
    ASDSL_CUDA(cudaMemcpy(w1, e->lm.w1, b1, cudaMemcpyDefault));
    return kOk;
}

int asdsl_b200_engine_read_buffer(asdsl_b200_engine* e, int which, void* host, size_t bytes) {
    ENG_READY(e);
    const asdsl_b200_engine_config& c = e->cfg;
    const size_t qd = static_cast<size_t>(c.num_heads) * c.head_dim, kvd = static_cast<size_t>(c.num_kv_heads) * c.head_dim;
    const void* src = nullptr;
    size_t n = 0;
    switch (which) {
        case 0: src = e->resid; n = 4ull * c.hidden_size; break;
        case 1: src = e->qkv; n = 4 * (qd + 2 * kvd); break;
        case 2: src = e->att; n = 4 * qd; break;
        case 3: src = e->h; n = 4ull * c.intermediate_size; break;
        case 4: src = e->logits; n = 4ull * c.vocab_size; break;
        case 5: src = e->kq; n = static_cast<size_t>(c.num_layers) * e->kv_codes_per_layer; break;
        case 6: src = e->vq; n = static_cast<size_t>(c.num_layers) * e->kv_codes_per_layer; break;
        case 7: src = e->ks; n = 4ull * c.num_layers * e->kv_scales_per_layer; break;
        case 8: src = e->vs; n = 4ull * c.num_layers * e->kv_scales_per_layer; break;
        default: return set_error(kEinval, "engine_read_buffer: unknown buffer");
    }
    if (!host) return set_error(kEinval, "engine_read_buffer: null pointer");
    if (bytes < n) return set_error(kEinval, "engine_read_buffer: buffer too small (" + std::to_string(n) + " bytes)");
    DeviceGuard dg(e->device);
    ASDSL_CUDA(cudaStreamSynchronize(e->stream));
    ASDSL_CUDA(cudaMemcpy(host, src, n, cudaMemcpyDeviceToHost));
    return kOk;
}

}  // extern "C"
