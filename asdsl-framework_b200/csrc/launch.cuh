// launch.cuh -- host-side planning and launch of the streaming GEMV family.
#pragma once

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
constexpr uint32_t kSmemBudget = 200 * 1024;
constexpr uint32_t kBarBytes = 2 * kMaxStages * 8;

inline uint32_t round_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

inline uint32_t xarea_bytes(int pro, int K, int gs) {
    const int ng = K / gs;
    if (pro == kProF32) return round_up(static_cast<uint32_t>((K + ng + kConsumerWarps) * 4), 128);
    return round_up(static_cast<uint32_t>(((K + 15) & ~15) + ng * 12 + kConsumerWarps * 4), 128);
}

struct StreamIn {
    const void* base;
    long long unit_bytes;
    long long total_bytes;
};

struct LaunchOpts {
    int max_ctas = 0;      // 0 = one CTA per SM
    bool pdl = false;      // programmatic dependent launch attribute
};

template <int FMT, int PRO, int EPI>
int launch_stream_gemv(const StreamIn* in, int n_streams, long long n_units, long long pair_unit_off,
                       GemvArgs ga, cudaStream_t stream, const LaunchOpts& opt = LaunchOpts()) {
    if (n_units <= 0) return kOk;
    if (n_units > 0x7fffffffLL) return set_error(kEinval, "too many rows");
    PipeArgs pa;
    std::memset(&pa, 0, sizeof(pa));
    pa.n_streams = n_streams;
    pa.n_units = static_cast<int>(n_units);
    pa.pair_unit_off = static_cast<int>(pair_unit_off);
    long long ub_sum = 0;
    for (int i = 0; i < n_streams; ++i) {
        if (!aligned16(in[i].base))
            return set_error(kEinval, "weight buffers must be 16-byte aligned device pointers");
        ub_sum += in[i].unit_bytes;
    }
    const int nseg = pair_unit_off > 0 ? 2 : 1;
    const int sms = sm_count();
    int grid = opt.max_ctas > 0 ? opt.max_ctas : sms;
    if (grid > n_units) grid = static_cast<int>(n_units);
    const long long per_cta = (n_units + grid - 1) / grid;

    const uint32_t xa = xarea_bytes(PRO, ga.K, ga.gs);
    long long cu = 12288 / (ub_sum > 0 ? ub_sum : 1);
    if (cu < 1) cu = 1;
    if (cu > per_cta) cu = per_cta;
    uint32_t seg_bytes = 0, stage_bytes = 0;
    int stages = 0;
    for (;;) {
        seg_bytes = 0;
        for (int i = 0; i < n_streams; ++i) {
            pa.s[i].region_off = seg_bytes;
            seg_bytes += round_up(static_cast<uint32_t>(cu * in[i].unit_bytes + 48), 16);
        }
        stage_bytes = seg_bytes * nseg;
        const long long avail = static_cast<long long>(kSmemBudget) - kBarBytes - xa;
        stages = avail > 0 ? static_cast<int>(avail / stage_bytes) : 0;
        if (stages > kMaxStages) stages = kMaxStages;
        if (stages >= 2 || cu == 1) break;
        cu = cu / 2 > 0 ? cu / 2 : 1;
    }
    if (stages < 2) return set_error(kEinval, "in_features too large for the shared-memory pipeline");
    for (int i = 0; i < n_streams; ++i) {
        pa.s[i].base = static_cast<const uint8_t*>(in[i].base);
        pa.s[i].unit_bytes = in[i].unit_bytes;
        pa.s[i].total_bytes = in[i].total_bytes;
    }
    pa.units_per_chunk = static_cast<int>(cu);
    pa.n_stages = stages;
    pa.seg_bytes = seg_bytes;
    pa.stage_bytes = stage_bytes;
    pa.xarea_off = kBarBytes;
    pa.stage_off = round_up(kBarBytes + xa, 128);
    const uint32_t smem = pa.stage_off + static_cast<uint32_t>(stages) * stage_bytes;

    ga.status = device_status_ptr();
    if (!ga.status) return set_error(kEcuda, "cannot resolve the device status word");

    auto kern = k_stream_gemv<FMT, PRO, EPI>;
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
    if (opt.pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    ASDSL_CUDA(cudaLaunchKernelEx(&cfg, kern, pa, ga));
    return kOk;
}

}  // namespace asdsl
