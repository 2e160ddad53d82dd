// launch.cuh -- host-side planning and launch of the streaming GEMV family.
#pragma once

#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "gemv_stream.cuh"

namespace asdsl {

// -------- error plumbing (thread-local message, status codes of the C ABI) --------
enum : int { kOk = 0, kEinval = 1, kErange = 2, kEcuda = 3, kEnccl = 4, kEtimeout = 5, kEnomem = 6 };

inline std::string& last_error_msg() {
    thread_local std::string msg;
    return msg;
}
inline int set_error(int code, const std::string& msg) {
    last_error_msg() = msg;
    return code;
}
inline int cuda_check(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return kOk;
    return set_error(kEcuda, std::string(what) + ": " + cudaGetErrorString(e));
}
#define ASDSL_CUDA(call)                                   \
    do {                                                   \
        int _rc = ::asdsl::cuda_check((call), #call);      \
        if (_rc != ::asdsl::kOk) return _rc;               \
    } while (0)

__device__ unsigned int g_status_word;  // kernels' bounded-wait status bits

inline unsigned int* device_status_ptr() {
    // one status word per device (module-scope __device__ variable)
    static unsigned int* ptrs[64] = {nullptr};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return nullptr;
    if (!ptrs[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
        ptrs[dev] = static_cast<unsigned int*>(p);
    }
    return ptrs[dev];
}

inline int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = n > 0 ? n : 148;
    }
    return cached[dev];
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// dynamic shared memory budget of one streaming-GEMV CTA
// shared-memory budget per CTA: kCtasPerSm CTAs must fit one SM (228 KB)
#ifndef ASDSL_SMEM_BUDGET_KB
// dynamic shared memory per CTA (of the 227 KB an sm_100a block may use)
#define ASDSL_SMEM_BUDGET_KB (224 / ASDSL_CTAS_PER_SM)
#endif
#ifndef ASDSL_CHUNK_KB
// bytes per pipeline stage; measured on B200 decode chains: 48 KB stages in a 224 KB budget
// beat 64 KB stages in 208 KB by ~4 %
#define ASDSL_CHUNK_KB 48
#endif
constexpr uint32_t kSmemBudget = ASDSL_SMEM_BUDGET_KB * 1024;
constexpr uint32_t kBarBytes = 512;  // full[kMaxStages] + empty[kMaxStages]
static_assert(kBarBytes >= 2 * kMaxStages * 8, "barrier area too small");

inline uint32_t round_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// process-wide number of the next streaming-GEMV launch (one counter for every template
// instantiation), carried into the timeline records
inline unsigned int next_launch_number() {
    static std::atomic<unsigned int> n{0};
    return n.fetch_add(1u, std::memory_order_relaxed);
}

// process-wide launch policy (asdsl_b200_set_launch_policy)
struct LaunchPolicy {
    int ctas_per_sm = kCtasPerSm;  // 1 leaves an SM slot free for the next kernel of a chain
    int pdl = 1;                   // programmatic dependent launch on every streaming GEMV
    int mma_min_tokens = 0;        // multi-token GEMVs from this many rows on the tensor cores (0 = never)
};
inline LaunchPolicy& launch_policy() {
    static LaunchPolicy p;
    return p;
}

struct StreamIn {
    const void* base;
    long long unit_bytes;
    long long total_bytes;
};

struct LaunchOpts {
    int max_ctas = 0;      // 0 = one CTA per SM
    bool pdl = false;      // programmatic dependent launch attribute
    int row_bytes = 0;     // row-major block formats: bytes of one row
    int chunk_target = ASDSL_CHUNK_KB * 1024;  // bytes per pipeline stage (all segments and streams)
    int k_parts = 0;       // K-split of every unit; 0 = the plan's own choice (plan_split)
};

// The chunk (units per pipeline stage) and K-split of launch_stream_gemv's plan for a GEMV of
// n_units units of unit_stage bytes (all streams and segments), before shared memory bounds the
// chunk.  The K-split fixes the order in which a row's slices are summed, so two launches that
// must give bit-identical rows (a single-token GEMV and a multi-token one over the same weights)
// pass the same k_parts.
struct PlanSplit {
    int grid;
    long long cu;
    int parts;
};
inline PlanSplit plan_split(long long n_units, long long unit_stage, int nseg, int rows_per_unit, int K,
                            const LaunchOpts& opt) {
    PlanSplit ps;
    ps.grid = opt.max_ctas > 0 ? opt.max_ctas : sm_count() * launch_policy().ctas_per_sm;
    if (ps.grid > n_units) ps.grid = static_cast<int>(n_units);
    if (ps.grid < 1) ps.grid = 1;
    const long long per_cta = (n_units + ps.grid - 1) / ps.grid;
    // stage = chunk of `cu` units (all segments and streams): big bulk copies stream
    // HBM best (>= 16 KB each), and every consumer warp shares every stage.
    ps.cu = opt.chunk_target / (unit_stage > 0 ? unit_stage : 1);
    if (ps.cu < 1) ps.cu = 1;
    if (ps.cu > per_cta) ps.cu = per_cta;
    // K-split so a chunk carries at least one work item per consumer warp
    ps.parts = 1;
    const int nq = K / 32;
    if (rows_per_unit == 4 && nq % 32 == 0 && ps.cu * nseg < kConsumerWarps) {
        // split K only when each part keeps >= 2 whole lane iterations (two slices in
        // flight); short rows are cheaper unsplit than merged through shared memory, even when
        // the CTA's whole share has fewer units than warps: measured on B200, parts of one lane
        // iteration for the 3072-row projections (3 x the items) made a decode step 6 % slower
        const int li = nq / 32;
        for (int d = 2; d <= 8 && d <= li; ++d) {
            if (li % d || li / d < 2) continue;
            ps.parts = d;
            if (ps.cu * nseg * d >= kConsumerWarps) break;
        }
    }
    return ps;
}

// Plan one GEMV of a persistent multi-op kernel whose ring has n_slots fixed slots of
// slot_bytes: the same chunking and K-split rules as launch_stream_gemv, with the chunk
// bounded by the slot.  Returns the bytes of K-split partials and counters the op needs.
inline int plan_ring_gemv(const StreamIn* in, int n_streams, long long n_units, long long pair_unit_off, int K,
                          int grid, uint32_t slot_bytes, int n_slots, int row_bytes, PipeArgs& pa,
                          uint32_t* part_bytes, uint32_t* cnt_bytes) {
    std::memset(&pa, 0, sizeof(pa));
    if (n_units <= 0 || n_units > 0x7fffffffLL) return set_error(kEinval, "plan_ring_gemv: bad unit count");
    pa.n_units = static_cast<int>(n_units);
    pa.pair_unit_off = static_cast<int>(pair_unit_off);
    long long ub_sum = 0;
    for (int i = 0; i < n_streams; ++i) {
        if (!aligned16(in[i].base)) return set_error(kEinval, "weight buffers must be 16-byte aligned device pointers");
        ub_sum += in[i].unit_bytes;
    }
    const int nseg = pair_unit_off > 0 ? 2 : 1;
    const long long per_cta = (n_units + grid - 1) / grid;
    long long cu = per_cta;
    for (;; --cu) {
        uint32_t seg = 0;
        for (int i = 0; i < n_streams; ++i) seg += round_up(static_cast<uint32_t>(cu * in[i].unit_bytes + 48), 16);
        if (static_cast<long long>(seg) * nseg <= slot_bytes || cu == 1) break;
    }
    int parts = 1;
    const int nq = K / 32;
    if (nq % 32 == 0 && cu * nseg < kConsumerWarps) {
        const int li = nq / 32;
        for (int d = 2; d <= 8 && d <= li; ++d) {
            if (li % d || li / d < 2) continue;
            parts = d;
            if (cu * nseg * d >= kConsumerWarps) break;
        }
    }
    uint32_t seg_bytes = 0;
    for (int i = 0; i < n_streams; ++i) {
        pa.s[i].base = static_cast<const uint8_t*>(in[i].base);
        pa.s[i].unit_bytes = in[i].unit_bytes;
        pa.s[i].total_bytes = in[i].total_bytes;
        pa.s[i].region_off = seg_bytes;
        seg_bytes += round_up(static_cast<uint32_t>(cu * in[i].unit_bytes + 48), 16);
    }
    if (static_cast<long long>(seg_bytes) * nseg > slot_bytes)
        return set_error(kEinval, "plan_ring_gemv: one unit does not fit a ring slot");
    const int ipu = parts * nseg;
    pa.units_per_chunk = static_cast<int>(cu);
    pa.n_stages = n_slots;
    pa.k_parts = parts;
    for (int p = 0; p <= parts; ++p) pa.q_bounds[p] = (nq / parts) * p;
    pa.inv_ipu = 1.0f / static_cast<float>(ipu);
    pa.seg_bytes = seg_bytes;
    pa.stage_bytes = seg_bytes * nseg;
    pa.row_bytes = row_bytes;
    *part_bytes = ipu > 1 ? round_up(static_cast<uint32_t>(n_slots * cu * ipu * 4 * 4), 16) : 0u;
    *cnt_bytes = ipu > 1 ? round_up(static_cast<uint32_t>(n_slots * cu * 4), 16) : 0u;
    return kOk;
}

template <int FMT, int PRO, int EPI, int NT = 1>
int launch_stream_gemv(const StreamIn* in, int n_streams, long long n_units, long long pair_unit_off,
                       GemvArgs ga, cudaStream_t stream, const LaunchOpts& opt = LaunchOpts()) {
    if (NT == 1) ga.n_tokens = 1;
    if (ga.n_tokens < 1 || ga.n_tokens > NT) return set_error(kEinval, "internal: token count out of range");
    if (n_units <= 0) return kOk;
    if (n_units > 0x7fffffffLL) return set_error(kEinval, "too many rows");
    PipeArgs pa;
    std::memset(&pa, 0, sizeof(pa));
    if (n_streams != FmtTraits<FMT>::kStreams) return set_error(kEinval, "internal: stream count mismatch");
    pa.n_units = static_cast<int>(n_units);
    pa.pair_unit_off = static_cast<int>(pair_unit_off);
    long long ub_sum = 0;
    for (int i = 0; i < n_streams; ++i) {
        if (!aligned16(in[i].base))
            return set_error(kEinval, "weight buffers must be 16-byte aligned device pointers");
        ub_sum += in[i].unit_bytes;
    }
    const int nseg = pair_unit_off > 0 ? 2 : 1;
    const LaunchPolicy pol = launch_policy();
    // kProRmsA8X also stages the fp32 activation behind its A8 area (the sequential norm chains)
    const uint32_t xa = xarea_layout_bytes(ga.K, ga.gs, PRO == kProF32) * static_cast<uint32_t>(ga.n_tokens) +
                        (PRO == kProRmsA8X ? 4u * static_cast<uint32_t>(ga.K) : 0u);
    const PlanSplit ps = plan_split(n_units, ub_sum * nseg, nseg, FmtTraits<FMT>::kRowsPerUnit, ga.K, opt);
    const int grid = ps.grid;
    long long cu = ps.cu;
    int parts = ps.parts;
    const int nq = ga.K / 32;
    if (is_exact_fmt(FMT)) {
        parts = 1;  // exact mode: each row's groups are summed in order by the threads of one warp
    } else if (opt.k_parts > 0) {
        // a forced split must cut K into parts of whole lane iterations (32 slices)
        if (opt.k_parts > 1 &&
            (opt.k_parts > 8 || nq % (32 * opt.k_parts) != 0 || FmtTraits<FMT>::kRowsPerUnit != 4))
            return set_error(kEinval, "internal: K-split does not divide in_features");
        parts = opt.k_parts;
    }
    const int ipu = parts * nseg;
    uint32_t seg_bytes = 0, stage_bytes = 0, split_bytes = 0;
    int stages = 0;
    for (;;) {
        seg_bytes = 0;
        for (int i = 0; i < n_streams; ++i) {
            pa.s[i].region_off = seg_bytes;
            seg_bytes += round_up(static_cast<uint32_t>(cu * in[i].unit_bytes + 48), 16);
        }
        stage_bytes = seg_bytes * nseg;
        split_bytes = 0;
        const long long avail = static_cast<long long>(kSmemBudget) - kBarBytes - xa;
        stages = avail > 0 ? static_cast<int>(avail / stage_bytes) : 0;
        if (stages > kMaxStages) stages = kMaxStages;
        if (ipu > 1 && stages > 0) {
            // partial sums + counters live beside the stages
            for (;;) {
                split_bytes = round_up(static_cast<uint32_t>(stages * cu * ipu * 4 * 4 * NT + stages * cu * 4), 128);
                if (stages <= 2 || static_cast<long long>(stages) * stage_bytes + split_bytes <= avail) break;
                --stages;
            }
        }
        if (stages >= 2 || cu == 1) break;
        cu = cu / 2 > 0 ? cu / 2 : 1;
    }
    if (stages < 2 || static_cast<long long>(stages) * stage_bytes + split_bytes >
                          static_cast<long long>(kSmemBudget) - kBarBytes - xa)
        return set_error(kEinval, "in_features too large for the shared-memory pipeline");
    for (int i = 0; i < n_streams; ++i) {
        pa.s[i].base = static_cast<const uint8_t*>(in[i].base);
        pa.s[i].unit_bytes = in[i].unit_bytes;
        pa.s[i].total_bytes = in[i].total_bytes;
    }
    pa.units_per_chunk = static_cast<int>(cu);
    pa.n_stages = stages;
    pa.k_parts = parts;
    {
        for (int p = 0; p <= parts; ++p) pa.q_bounds[p] = (nq / parts) * p;
        pa.inv_ipu = 1.0f / static_cast<float>(ipu);
    }
    pa.seg_bytes = seg_bytes;
    pa.stage_bytes = stage_bytes;
    pa.xarea_off = kBarBytes;
    pa.stage_off = round_up(kBarBytes + xa, 128);
    pa.split_off = pa.stage_off + static_cast<uint32_t>(stages) * stage_bytes;
    pa.row_bytes = opt.row_bytes;
    if (PRO != kProQ8 && !aligned16(ga.x)) return set_error(kEinval, "activations must be 16-byte aligned");
    if (pro_is_rms(PRO) && !aligned16(ga.norm_w)) return set_error(kEinval, "norm weights must be 16-byte aligned");
    if (PRO == kProQ8 && (reinterpret_cast<uintptr_t>(ga.xq) & 3u))
        return set_error(kEinval, "int8 activations must be 4-byte aligned");
    const uint32_t smem = pa.split_off + split_bytes;

    ga.status = device_status_ptr();
    if (!ga.status) return set_error(kEcuda, "cannot resolve the device status word");
    ga.tl_id = next_launch_number();

    auto kern = k_stream_gemv<FMT, PRO, EPI, NT>;
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
    if (opt.pdl || pol.pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    ASDSL_CUDA(cudaLaunchKernelEx(&cfg, kern, pa, ga));
    return kOk;
}

// Exact-mode GEMV over preq2 weights (reference-exact numerics): rows [0, M) of meta / quant, or
// the paired gate/up form (pair_rows = I: gate rows [0, I), up rows [I, 2I)).  A unit is L bands;
// large row counts use more lanes per thread (fewer instructions per row), small ones fewer (more
// threads per row).  ASDSL_EXACT_LPT = 1, 2, 4 or 8 forces the choice.
inline int exact_lpt_for(long long m_seg, bool pair) {
    const long long nb_seg = (m_seg + 3) / 4;
    // a paired (gate/up) unit is computed by one warp in two passes: rank it by one half's rows
    const long long work_rows = m_seg;
    // measured in the config-3 exact decode chain (B200): 3072- and 5120-row matrices run 1.5 %
    // faster per token with 2 lanes per thread than with 1, the 200064-row lm_head 0.7 % faster
    // with 4 than with 8; 16384-row matrices are fastest with 4 (back-to-back launches)
    int lpt = work_rows >= 14208 ? 4 : (work_rows >= 3072 ? 2 : 1);
    static const int forced = [] {
        const char* v = std::getenv("ASDSL_EXACT_LPT");
        const int f = v ? std::atoi(v) : 0;
        return (f == 1 || f == 2 || f == 4 || f == 8) ? f : 0;
    }();
    if (forced) lpt = forced;
    while (lpt > 1 && pair && nb_seg % lpt) lpt >>= 1;  // the up segment starts on a unit
    return lpt;
}

// inter_lpt = 0: meta / quant are the reference's preq2 bytes; > 0: they are in the exact layout
// of k_relayout_exact with units of inter_lpt bands.
template <int PRO, int EPI>
int launch_exact_gemv(const uint8_t* meta, const uint8_t* quant, long long M_total, long long pair_rows, GemvArgs ga,
                      cudaStream_t stream, int inter_lpt = 0) {
    const long long K = ga.K;
    const long long ng = K / 32;
    const long long m_seg = pair_rows > 0 ? pair_rows : M_total;
    const long long nb_seg = (m_seg + 3) / 4;
    const long long nb_all = (M_total + 3) / 4;
    const int lpt = inter_lpt > 0 ? inter_lpt : exact_lpt_for(m_seg, pair_rows > 0);
    if (pair_rows > 0 && nb_seg % lpt) return set_error(kEinval, "internal: exact gate/up units straddle the halves");
    StreamIn in[2];
    if (inter_lpt > 0) {
        const long long units_all = (nb_all + lpt - 1) / lpt;
        in[0] = StreamIn{quant, ng * 64 * lpt, units_all * ng * 64 * lpt};
        in[1] = StreamIn{meta, ng * 16 * lpt, units_all * ng * 16 * lpt};
    } else {
        in[0] = StreamIn{quant, ng * 64 * lpt, nb_all * ng * 64};
        in[1] = StreamIn{meta, ng * 16 * lpt, M_total * ng * 4};
    }
    const long long nu = (nb_seg + lpt - 1) / lpt;
    const long long off = pair_rows > 0 ? nb_seg / lpt : 0;
    ga.gs = 32;
    ga.exact_inter = inter_lpt > 0 ? 1 : 0;
    switch (lpt) {
        case 8: return launch_stream_gemv<kFmtPreq2X8, PRO, EPI>(in, 2, nu, off, ga, stream);
        case 4: return launch_stream_gemv<kFmtPreq2X4, PRO, EPI>(in, 2, nu, off, ga, stream);
        case 2: return launch_stream_gemv<kFmtPreq2X2, PRO, EPI>(in, 2, nu, off, ga, stream);
        default: return launch_stream_gemv<kFmtPreq2X, PRO, EPI>(in, 2, nu, off, ga, stream);
    }
}

}  // namespace asdsl
