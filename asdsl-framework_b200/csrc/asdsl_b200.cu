// asdsl_b200.cu -- the C ABI of the B200-native ASDSL decode hot path.
//
// Single translation unit: the kernel headers are included here so that the
// library needs no relocatable device code.  Every exported function is
// declared in include/asdsl_b200.h with the reference interface it replaces.
#include "../../include/asdsl_b200.h"

#include <utility>
#include <vector>

#include "launch.cuh"
#include "weight_prep.cuh"
#include "gemv_mma.cuh"
#include "gemv_q2.cuh"
#include "gemm_q4_128.cuh"

using namespace asdsl;

namespace {

constexpr int kMaxK = 20480;  // reference thread_local A8 scratch (gemv_preq2_avx2.cpp:315-316)

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// ---------------------------------------------------------------------------
// standalone A8 (quantize_activation_avx2): one warp per group, any group size
// ---------------------------------------------------------------------------
__global__ void k_quantize_activation(const float* __restrict__ x, int8_t* __restrict__ xq, float* __restrict__ xs,
                                      int32_t* __restrict__ xsum, int K, int gs) {
    const int wpb = blockDim.x >> 5;
    const int g = blockIdx.x * wpb + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const int ng = K / gs;
    if (g >= ng) return;
    const float* xg = x + static_cast<long long>(g) * gs;
    float amax = 0.0f;
    for (int j = lane; j < gs; j += 32) amax = fmaxf(amax, fabsf(xg[j]));
    amax = warp_max(amax);
    int8_t* q = xq + static_cast<long long>(g) * gs;
    int s = 0;
    if (amax < 1e-9f) {
        for (int j = lane; j < gs; j += 32) q[j] = 0;
        if (lane == 0) xs[g] = 1.0f;
    } else {
        const float inv = __fdiv_rn(127.0f, amax);
        for (int j = lane; j < gs; j += 32) {
            const int c = a8_code(xg[j], inv);
            q[j] = static_cast<int8_t>(c);
            s += c;
        }
        if (lane == 0) xs[g] = __fmul_rn(amax, inv127f());
    }
    s = warp_sum_i(s);
    if (xsum && lane == 0) xsum[g] = s;
}

// ---------------------------------------------------------------------------
// unpacked (one code per byte) fp32-activation GEMV: warp per row, lane per group
// (gemv_q4_avx2.cpp:755-806; a compatibility path, not the decode hot path)
// ---------------------------------------------------------------------------
__global__ void k_gemv_unpacked(const uint8_t* __restrict__ w, const float* __restrict__ x,
                                const float* __restrict__ scales, const float* __restrict__ biases,
                                float* __restrict__ y, int M, int K, int gs) {
    const int wpb = blockDim.x >> 5;
    const int row = blockIdx.x * wpb + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= M) return;
    const int ng = K / gs;
    const uint8_t* wr = w + static_cast<long long>(row) * K;
    float acc = 0.0f;
    for (int g = lane; g < ng; g += 32) {
        float d = 0.0f, sx = 0.0f;
        for (int j = 0; j < gs; ++j) {
            const float xv = x[g * gs + j];
            d = __fmaf_rn(static_cast<float>(wr[g * gs + j]), xv, d);
            sx = __fadd_rn(sx, xv);
        }
        const long long gi = static_cast<long long>(row) * ng + g;
        acc += __fmaf_rn(d, scales[gi], __fmul_rn(biases[gi], sx));
    }
    acc = warp_sum(acc);
    if (lane == 0) y[row] = acc;
}

int check_k(int K, int gs, const char* fn) {
    if (gs <= 0 || K <= 0) return set_error(kEinval, std::string(fn) + ": invalid dimensions");
    if (K % gs != 0) return set_error(kEinval, std::string(fn) + ": in_features must be divisible by group_size");
    if (K > kMaxK) return set_error(kEinval, std::string(fn) + ": n_groups exceeds buffer");
    return kOk;
}

// preq2 streams: quant (band units) + meta (4 rows per band)
inline void preq2_streams(StreamIn* s, const uint8_t* meta, const uint8_t* quant, long long M, long long K) {
    const long long ng = K / 32;
    const long long nb = (M + 3) / 4;
    s[0] = StreamIn{quant, ng * 64, nb * ng * 64};
    s[1] = StreamIn{meta, ng * 16, M * ng * 4};
}

LaunchOpts rows_opt(long long row_bytes) {
    LaunchOpts o;
    o.row_bytes = static_cast<int>(row_bytes);
    return o;
}

// banded Q4_128 streams: quant [nb][ng][4][64] + scales [nb][ng][4] fp16 (band units)
inline void q128b_streams(StreamIn* s, const uint8_t* quant, const uint8_t* scales, long long M, long long K) {
    const long long ng = K / 128;
    const long long nb = (M + 3) / 4;
    s[0] = StreamIn{quant, ng * 256, nb * ng * 256};
    s[1] = StreamIn{scales, ng * 8, nb * ng * 8};
}

int check_k128(int K, const char* fn) {
    if (K <= 0 || K % 128) return set_error(kEinval, std::string(fn) + ": in_features must be divisible by 128");
    if (K > 17920) return set_error(kEinval, std::string(fn) + ": in_features exceeds 17920");
    return kOk;
}

GemvArgs base_args(int M, int K, int gs) {
    GemvArgs ga;
    std::memset(&ga, 0, sizeof(ga));
    ga.M = M;
    ga.K = K;
    ga.gs = gs;
    return ga;
}

}  // namespace

// ===========================================================================
// exported C ABI
// ===========================================================================
extern "C" {

const char* asdsl_b200_version(void) { return "asdsl-b200 0.1 (sm_100a)"; }

const char* asdsl_b200_last_error(void) { return last_error_msg().c_str(); }

int asdsl_b200_set_mma_min_tokens(int n_tokens) {
    if (n_tokens < 0) return set_error(kEinval, "set_mma_min_tokens: negative token count");
    launch_policy().mma_min_tokens = n_tokens;
    return kOk;
}

int asdsl_b200_set_launch_policy(int ctas_per_sm, int use_pdl) {
    if (ctas_per_sm < 1 || ctas_per_sm > kCtasPerSm)
        return set_error(kEinval, "set_launch_policy: ctas_per_sm must be in [1, " + std::to_string(kCtasPerSm) + "]");
    launch_policy().ctas_per_sm = ctas_per_sm;
    launch_policy().pdl = use_pdl ? 1 : 0;
    return kOk;
}

int asdsl_b200_device_status(unsigned int* status, int clear) {
    if (!status) return set_error(kEinval, "asdsl_b200_device_status: null pointer");
    ASDSL_CUDA(cudaDeviceSynchronize());
    unsigned int v = 0;
    ASDSL_CUDA(cudaMemcpyFromSymbol(&v, g_status_word, sizeof(v)));
    *status = v;
    if (clear) {
        const unsigned int z = 0;
        ASDSL_CUDA(cudaMemcpyToSymbol(g_status_word, &z, sizeof(z)));
    }
    return kOk;
}

int asdsl_b200_timeline_set(void* buf, unsigned int slots_per_block) {
    if (!kTimeline && buf != nullptr)
        return set_error(kEinval, "timeline_set: this library was built without timeline records; load "
                                  "libasdsl_b200_timeline.so (set ASDSL_B200_TIMELINE=1 before loading asdsl_b200)");
    if (buf != nullptr && (slots_per_block == 0 || (reinterpret_cast<uintptr_t>(buf) & 15u)))
        return set_error(kEinval, "timeline_set: need a 16-byte aligned device buffer and a slot count");
    ASDSL_CUDA(cudaDeviceSynchronize());
    // buffer: [kTlMaxBlocks] uint32 slot counters, then the records [kTlMaxBlocks][slots][kTlEvents]
    uint32_t* cnt = static_cast<uint32_t*>(buf);
    TlRec* recs = buf ? reinterpret_cast<TlRec*>(static_cast<uint8_t*>(buf) + 4 * kTlMaxBlocks) : nullptr;
    const uint32_t slots = buf ? slots_per_block : 0u;
    if (buf) ASDSL_CUDA(cudaMemset(buf, 0, 4 * kTlMaxBlocks));
    ASDSL_CUDA(cudaMemcpyToSymbol(g_tl_cnt, &cnt, sizeof(cnt)));
    ASDSL_CUDA(cudaMemcpyToSymbol(g_tl_slots, &slots, sizeof(slots)));
    ASDSL_CUDA(cudaMemcpyToSymbol(g_tl_buf, &recs, sizeof(recs)));
    return kOk;
}

size_t asdsl_b200_timeline_bytes(unsigned int slots_per_block) {
    return 4ull * kTlMaxBlocks + sizeof(TlRec) * kTlEvents * static_cast<size_t>(kTlMaxBlocks) * slots_per_block;
}

int asdsl_b200_quantize_activation(const float* x, int8_t* xq, float* xs, int32_t* xsum, int K, int gs,
                                   void* stream) {
    if (!x || !xq || !xs) return set_error(kEinval, "quantize_activation: null pointer");
    if (gs <= 0 || K < 0) return set_error(kEinval, "quantize_activation: invalid dimensions");
    const int ng = K / gs;
    if (ng == 0) return kOk;
    const int wpb = 8;
    k_quantize_activation<<<(ng + wpb - 1) / wpb, wpb * 32, 0, as_stream(stream)>>>(x, xq, xs, xsum, K, gs);
    ASDSL_CUDA(cudaGetLastError());
    return kOk;
}

int asdsl_b200_gemv_preq2_fused(const uint8_t* meta, const uint8_t* quant, const float* x, float* y, int M, int K,
                                int gs, void* stream) {
    if (!meta || !quant || !x || !y) return set_error(kEinval, "gemv_preq2_fused_avx2: null pointer");
    if (gs != 32) return set_error(kEinval, "gemv_preq2_fused_avx2: group_size must be 32");
    if (int rc = check_k(K, gs, "gemv_preq2_fused_avx2")) return rc;
    if (M < 0) return set_error(kEinval, "gemv_preq2_fused_avx2: invalid dimensions");
    StreamIn s[2];
    preq2_streams(s, meta, quant, M, K);
    GemvArgs ga = base_args(M, K, 32);
    ga.x = x;
    ga.y = y;
    return launch_stream_gemv<kFmtPreq2, kProA8, kEpiStore>(s, 2, (M + 3) / 4, 0, ga, as_stream(stream));
}

int asdsl_b200_gemv_preq2(const uint8_t* meta, const uint8_t* quant, const int8_t* xq, const float* xs, float* y,
                          int M, int K, int gs, void* stream) {
    if (!meta || !quant || !xq || !xs || !y) return set_error(kEinval, "gemv_preq2_avx2: null pointer");
    if (gs != 32) return set_error(kEinval, "gemv_preq2_avx2: group_size must be 32");
    if (int rc = check_k(K, gs, "gemv_preq2_avx2")) return rc;
    if (M < 0) return set_error(kEinval, "gemv_preq2_avx2: invalid dimensions");
    StreamIn s[2];
    preq2_streams(s, meta, quant, M, K);
    GemvArgs ga = base_args(M, K, 32);
    ga.xq = xq;
    ga.xs_in = xs;
    ga.y = y;
    return launch_stream_gemv<kFmtPreq2, kProQ8, kEpiStore>(s, 2, (M + 3) / 4, 0, ga, as_stream(stream));
}

int asdsl_b200_gemv_q4_32_preq(const uint8_t* blocks, const int8_t* xq, const float* xs, float* y, int M, int K,
                               int gs, void* stream) {
    if (!blocks || !xq || !xs || !y) return set_error(kEinval, "gemv_q4_32_preq_avx2: null input pointer");
    if (M <= 0 || K <= 0 || gs <= 0) return set_error(kEinval, "gemv_q4_32_preq_avx2: invalid dimensions");
    if (K % gs) return set_error(kEinval, "gemv_q4_32_preq_avx2: in_features must be divisible by group_size");
    if (gs != 32) return set_error(kEinval, "gemv_q4_32_preq_avx2: group_size must be 32");
    if (K / gs > 640) return set_error(kEinval, "gemv_q4_32_preq_avx2: n_groups exceeds buffer");
    const long long ng = K / 32;
    StreamIn s[1] = {{blocks, 4 * ng * 20, static_cast<long long>(M) * ng * 20}};
    GemvArgs ga = base_args(M, K, 32);
    ga.xq = xq;
    ga.xs_in = xs;
    ga.y = y;
    return launch_stream_gemv<kFmtPreq, kProQ8, kEpiStore>(s, 1, (M + 3) / 4, 0, ga, as_stream(stream),
                                                           rows_opt(ng * 20));
}

int asdsl_b200_gemv_q4_32_preq_fused(const uint8_t* blocks, const float* x, float* y, int M, int K, int gs,
                                     void* stream) {
    if (!blocks || !x || !y) return set_error(kEinval, "gemv_q4_32_preq_fused_avx2: null input pointer");
    if (gs != 32) return set_error(kEinval, "gemv_q4_32_preq_fused_avx2: group_size must be 32");
    if (M <= 0 || K <= 0) return set_error(kEinval, "gemv_q4_32_preq_fused_avx2: invalid dimensions");
    if (int rc = check_k(K, gs, "gemv_q4_32_preq_fused_avx2")) return rc;
    const long long ng = K / 32;
    StreamIn s[1] = {{blocks, 4 * ng * 20, static_cast<long long>(M) * ng * 20}};
    GemvArgs ga = base_args(M, K, 32);
    ga.x = x;
    ga.y = y;
    return launch_stream_gemv<kFmtPreq, kProA8, kEpiStore>(s, 1, (M + 3) / 4, 0, ga, as_stream(stream),
                                                           rows_opt(ng * 20));
}

int asdsl_b200_gemv_q4_128(const uint8_t* blocks, const int8_t* xq, const float* xs, float* y, int M, int K, int gs,
                           void* stream) {
    if (!blocks || !xq || !xs || !y) return set_error(kEinval, "gemv_q4_128_preq_avx2: null pointer");
    if (gs != 128) return set_error(kEinval, "gemv_q4_128_preq_avx2: group_size must be 128");
    if (K <= 0 || K % 128) return set_error(kEinval, "gemv_q4_128_preq_avx2: in_features must be divisible by 128");
    if (K > 17920) return set_error(kEinval, "gemv_q4_128_preq_avx2: in_features exceeds 17920");
    if (M < 0) return set_error(kEinval, "gemv_q4_128_preq_avx2: invalid dimensions");
    const long long ng = K / 128;
    StreamIn s[1] = {{blocks, 4 * ng * 66, static_cast<long long>(M) * ng * 66}};
    GemvArgs ga = base_args(M, K, 128);
    ga.xq = xq;
    ga.xs_in = xs;
    ga.y = y;
    return launch_stream_gemv<kFmtQ4_128, kProQ8, kEpiStore>(s, 1, (M + 3) / 4, 0, ga, as_stream(stream),
                                                             rows_opt(ng * 66));
}

int asdsl_b200_gemm_q4_128_f32(const uint8_t* blocks, const float* X, float* Y, int M, int K, int gs, int batch,
                               void* stream) {
    if (gs != 128) return set_error(kEinval, "gemm_q4_128_q8_avx2: group_size must be 128");
    if (!blocks || !X || !Y) return set_error(kEinval, "gemm_q4_128_q8_avx2: null pointer");
    if (K <= 0 || K % 128) return set_error(kEinval, "gemm_q4_128_q8_avx2: in_features must be divisible by 128");
    if (M < 0 || batch < 0) return set_error(kEinval, "gemm_q4_128_q8_avx2: invalid dimensions");
    if (reinterpret_cast<uintptr_t>(blocks) & 1u) return set_error(kEinval, "gemm_q4_128_q8_avx2: blocks must be 2-byte aligned");
    if (!aligned16(X)) return set_error(kEinval, "gemm_q4_128_q8_avx2: activations must be 16-byte aligned");
    const int B = batch < asdsl::kGemmMaxBatch ? batch : asdsl::kGemmMaxBatch;  // the reference stops at 64
    if (M == 0 || B == 0) return kOk;
    static std::mutex mu;
    static bool configured[64] = {false};
    int dev = 0;
    ASDSL_CUDA(cudaGetDevice(&dev));
    {
        std::lock_guard<std::mutex> lk(mu);
        if (dev >= 0 && dev < 64 && !configured[dev]) {
            ASDSL_CUDA(cudaFuncSetAttribute(asdsl::k_gemm_q4_128_f32, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(asdsl::kGemmSmem)));
            configured[dev] = true;
        }
    }
    const unsigned grid = static_cast<unsigned>((M + asdsl::kGemmRows - 1) / asdsl::kGemmRows);
    asdsl::k_gemm_q4_128_f32<<<grid, 256, asdsl::kGemmSmem, as_stream(stream)>>>(blocks, X, Y, M, K, B);
    ASDSL_CUDA(cudaGetLastError());
    return kOk;
}

int asdsl_b200_gemv_q4_128_fused(const uint8_t* blocks, const float* x, float* y, int M, int K, void* stream) {
    if (!blocks || !x || !y) return set_error(kEinval, "gemv_q4_128_fused: null pointer");
    if (K <= 0 || K % 128) return set_error(kEinval, "gemv_q4_128_fused: in_features must be divisible by 128");
    if (K > 17920) return set_error(kEinval, "gemv_q4_128_fused: in_features exceeds 17920");
    if (M < 0) return set_error(kEinval, "gemv_q4_128_fused: invalid dimensions");
    const long long ng = K / 128;
    StreamIn s[1] = {{blocks, 4 * ng * 66, static_cast<long long>(M) * ng * 66}};
    GemvArgs ga = base_args(M, K, 128);
    ga.x = x;
    ga.y = y;
    return launch_stream_gemv<kFmtQ4_128, kProA8, kEpiStore>(s, 1, (M + 3) / 4, 0, ga, as_stream(stream),
                                                             rows_opt(ng * 66));
}

int asdsl_b200_gemv_q4_s256(const uint8_t* blocks, const int8_t* xq, const float* xs, float* y, int M, int K, int gs,
                            void* stream) {
    if (!blocks || !xq || !xs || !y) return set_error(kEinval, "gemv_q4_s256: null pointer");
    if (gs != 32) return set_error(kEinval, "gemv_q4_s256: group_size must be 32");
    if (K <= 0 || K % 256) return set_error(kEinval, "gemv_q4_s256: in_features must be divisible by 256");
    if (K > 17920) return set_error(kEinval, "gemv_q4_s256: in_features exceeds 17920");
    if (M < 0) return set_error(kEinval, "gemv_q4_s256: invalid dimensions");
    const long long nsb = K / 256;
    StreamIn s[1] = {{blocks, 4 * nsb * 144, static_cast<long long>(M) * nsb * 144}};
    GemvArgs ga = base_args(M, K, 32);
    ga.xq = xq;
    ga.xs_in = xs;
    ga.y = y;
    return launch_stream_gemv<kFmtS256, kProQ8, kEpiStore>(s, 1, (M + 3) / 4, 0, ga, as_stream(stream),
                                                           rows_opt(nsb * 144));
}

int asdsl_b200_gemv_q4km(const uint8_t* w, const float* x, float* y, int M, int K, void* stream) {
    if (K <= 0 || M <= 0) return kOk;  // the reference returns without work (gemv_q4_avx2.cpp:364-366)
    if (!w || !x || !y) return set_error(kEinval, "gemv_q4km_q8_avx2: null pointer");
    if (K % 256) return set_error(kEinval, "in_features must be divisible by 256 for Q4_K_M");
    if (K > kMaxK) return set_error(kEinval, "gemv_q4km_q8_avx2: in_features too large");
    const long long nb = K / 256;
    StreamIn s[1] = {{w, 4 * nb * 144, static_cast<long long>(M) * nb * 144}};
    GemvArgs ga = base_args(M, K, 32);
    ga.x = x;
    ga.y = y;
    return launch_stream_gemv<kFmtQ4K, kProQ4K, kEpiStore>(s, 1, (M + 3) / 4, 0, ga, as_stream(stream),
                                                           rows_opt(nb * 144));
}

int asdsl_b200_gemv_q4_packed(const uint8_t* w, const float* x, const float* scales, const float* biases, float* y,
                              int M, int K, int gs, int batch, void* stream) {
    if (!w || !x || !scales || !biases || !y) return set_error(kEinval, "gemv_q4_packed: null pointer");
    if (M <= 0 || K <= 0 || gs <= 0) return set_error(kEinval, "M, K, group_size must be positive");
    if (batch < 1) return set_error(kEinval, "batch must be >= 1");
    if (K % 2) return set_error(kEinval, "K must be even for 4-bit packing");
    if (K % gs) return set_error(kEinval, "K must be divisible by group_size");
    if (gs % 8) return set_error(kEinval, "group_size must be a multiple of 8 for AVX2 vectorization");
    if (K > 32768) return set_error(kEinval, "gemv_q4_packed: in_features too large");
    const long long ng = K / gs;
    StreamIn s[3] = {{w, K / 2, static_cast<long long>(M) * (K / 2)},
                     {scales, ng * 4, static_cast<long long>(M) * ng * 4},
                     {biases, ng * 4, static_cast<long long>(M) * ng * 4}};
    for (int b = 0; b < batch; ++b) {
        GemvArgs ga = base_args(M, K, gs);
        ga.x = x + static_cast<long long>(b) * K;
        ga.y = y + static_cast<long long>(b) * M;
        int rc = launch_stream_gemv<kFmtPacked, kProF32, kEpiStore>(s, 3, M, 0, ga, as_stream(stream));
        if (rc) return rc;
    }
    return kOk;
}

int asdsl_b200_gemv_q4_unpacked(const uint8_t* w, const float* x, const float* scales, const float* biases, float* y,
                                int M, int K, int gs, void* stream) {
    if (!w || !x || !scales || !biases || !y) return set_error(kEinval, "gemv_q4_unpacked: null pointer");
    if (M <= 0 || K <= 0 || gs <= 0) return set_error(kEinval, "M, K, group_size must be positive");
    if (K % 2) return set_error(kEinval, "K must be even for 4-bit packing");
    if (K % gs) return set_error(kEinval, "K must be divisible by group_size");
    if (gs % 8) return set_error(kEinval, "group_size must be a multiple of 8 for AVX2 vectorization");
    const int wpb = 8;
    k_gemv_unpacked<<<(M + wpb - 1) / wpb, wpb * 32, 0, as_stream(stream)>>>(w, x, scales, biases, y, M, K, gs);
    ASDSL_CUDA(cudaGetLastError());
    return kOk;
}

namespace {
int gemv_q2_impl(bool packed, const uint8_t* w, const float* x, const float* scales, const float* biases, float* y,
                 int M, int K, int gs, void* stream, const char* fn) {
    if (!w || !x || !scales || !biases || !y) return set_error(kEinval, std::string(fn) + ": null pointer");
    if (M <= 0 || K <= 0 || gs <= 0) return set_error(kEinval, "M, K, group_size must be positive");
    if (packed && K % 4) return set_error(kEinval, "K must be divisible by 4 for 2-bit packing");
    if (K % gs) return set_error(kEinval, "K must be divisible by group_size");
    if (packed && gs % 4) return set_error(kEinval, std::string(fn) + ": group_size must be a multiple of 4");
    if (K > 32768) return set_error(kEinval, std::string(fn) + ": in_features exceeds 32768");
    const size_t smem = 4ull * (K + K / gs);
    const void* fnp = packed ? reinterpret_cast<const void*>(&asdsl::k_gemv_q2<true>)
                             : reinterpret_cast<const void*>(&asdsl::k_gemv_q2<false>);
    if (smem > 48 * 1024)
        ASDSL_CUDA(cudaFuncSetAttribute(fnp, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    const unsigned grid = static_cast<unsigned>(
        std::min<long long>((M + asdsl::kQ2Warps - 1) / asdsl::kQ2Warps, sm_count() * 2ll));  // x staged once per CTA
    if (packed)
        asdsl::k_gemv_q2<true><<<grid, asdsl::kQ2Warps * 32, smem, as_stream(stream)>>>(w, x, scales, biases, y, M, K, gs,
                                                                                      0);
    else
        asdsl::k_gemv_q2<false><<<grid, asdsl::kQ2Warps * 32, smem, as_stream(stream)>>>(w, x, scales, biases, y, M, K,
                                                                                       gs, 0);
    ASDSL_CUDA(cudaGetLastError());
    return kOk;
}
}  // namespace

int asdsl_b200_gemv_q2_packed(const uint8_t* w_packed, const float* x, const float* scales, const float* biases,
                              float* y, int M, int K, int gs, void* stream) {
    return gemv_q2_impl(true, w_packed, x, scales, biases, y, M, K, gs, stream, "gemv_q2_packed");
}

int asdsl_b200_gemv_q2_unpacked(const uint8_t* w, const float* x, const float* scales, const float* biases, float* y,
                                int M, int K, int gs, void* stream) {
    return gemv_q2_impl(false, w, x, scales, biases, y, M, K, gs, stream, "gemv_q2_unpacked");
}

int asdsl_b200_matmul_batch_q4(const uint8_t* w, const float* scales, const float* biases, const float* X, float* Y,
                               int M, int K, int B, int gs, void* stream) {
    return asdsl_b200_gemv_q4_packed(w, X, scales, biases, Y, M, K, gs, B, stream);
}

size_t asdsl_b200_argmax_scratch_bytes(void) { return 256 + 2 * 4 * 1024; }

int asdsl_b200_relayout_q4_128(const uint8_t* blocks, uint8_t* quant, uint8_t* scales, int M, int K, void* stream) {
    if (!blocks || !quant || !scales) return set_error(kEinval, "relayout_q4_128: null pointer");
    if (int rc = check_k128(K, "relayout_q4_128")) return rc;
    if (M <= 0) return set_error(kEinval, "relayout_q4_128: invalid dimensions");
    const long long work = (static_cast<long long>(M) + 3) / 4 * (K / 128) * 4;
    const int threads = 256;
    long long blocks_n = (work + threads - 1) / threads;
    if (blocks_n > 65535) blocks_n = 65535;
    k_relayout_q4_128<<<static_cast<unsigned>(blocks_n), threads, 0, as_stream(stream)>>>(blocks, quant, scales, M, K);
    ASDSL_CUDA(cudaGetLastError());
    return kOk;
}

int asdsl_b200_gemv_q4_128_banded(const uint8_t* quant, const uint8_t* scales, const float* x, float* y, int M, int K,
                                  void* stream) {
    if (!quant || !scales || !x || !y) return set_error(kEinval, "gemv_q4_128_banded: null pointer");
    if (int rc = check_k128(K, "gemv_q4_128_banded")) return rc;
    if (M < 0) return set_error(kEinval, "gemv_q4_128_banded: invalid dimensions");
    StreamIn s[2];
    q128b_streams(s, quant, scales, M, K);
    GemvArgs ga = base_args(M, K, 128);
    ga.x = x;
    ga.y = y;
    return launch_stream_gemv<kFmtQ128B, kProA8, kEpiStore>(s, 2, (M + 3) / 4, 0, ga, as_stream(stream));
}

}  // extern "C"

// cross-GPU argmax exchange of a row-sharded lm_head (asdsl_b200_xchg_*)
struct asdsl_b200_xchg {
    int world = 1, rank = 0, device = 0;
    unsigned long long* slots = nullptr;       // this rank's [2][world] words
    int* epoch = nullptr;                      // device-resident step counter
    unsigned long long** peer_table = nullptr; // device array [world]
    void* mapped[64] = {};                     // opened peer mappings (null for self)
    bool open = false;
    unsigned long long* stamps = nullptr;      // optional %globaltimer stamps [n][4] (caller's memory)
    int stamp_mask = 0;
};

namespace {
int gemv_argmax_impl(int fmt, const uint8_t* w0, const uint8_t* w1, const float* x, float* y, float* out_val,
                     int32_t* out_idx, int row_base, void* scratch, size_t scratch_bytes, int M, int K, void* stream,
                     const asdsl_b200_xchg* xg) {
    if (!w0 || !x || !out_val || !out_idx || !scratch) return set_error(kEinval, "gemv_argmax: null pointer");
    if (scratch_bytes < asdsl_b200_argmax_scratch_bytes()) return set_error(kEinval, "gemv_argmax: scratch too small");
    if (M <= 0) return set_error(kEinval, "gemv_argmax: invalid dimensions");
    // the scratch holds one (value, index) pair per CTA of the grid, at fixed 1024-entry offsets
    if (static_cast<long long>(sm_count()) * launch_policy().ctas_per_sm > 1024)
        return set_error(kErange, "gemv_argmax: the grid exceeds the scratch layout's 1024 CTAs");
    uint8_t* sc = static_cast<uint8_t*>(scratch);
    GemvArgs ga;
    StreamIn s[2];
    auto finish = [&](GemvArgs& a) {
        a.x = x;
        a.y = y;
        a.counter = reinterpret_cast<unsigned int*>(sc);
        a.part_val = reinterpret_cast<float*>(sc + 256);
        a.part_idx = reinterpret_cast<int*>(sc + 256 + 4 * 1024);
        a.out_val = out_val;
        a.out_idx = out_idx;
        a.row_base = row_base;
        if (xg) {
            a.xchg_peers = xg->peer_table;
            a.xchg_self = xg->slots;
            a.xchg_epoch = xg->epoch;
            a.xchg_world = xg->world;
            a.xchg_rank = xg->rank;
            a.xchg_stamps = xg->stamps;
            a.xchg_stamp_mask = xg->stamp_mask;
        }
    };
    const long long nbands = (static_cast<long long>(M) + 3) / 4;
    if (fmt == ASDSL_B200_FMT_PREQ2) {
        if (!w1) return set_error(kEinval, "gemv_argmax: null pointer");
        if (int rc = check_k(K, 32, "gemv_argmax")) return rc;
        preq2_streams(s, w0, w1, M, K);
        ga = base_args(M, K, 32);
        finish(ga);
        return launch_stream_gemv<kFmtPreq2, kProA8, kEpiArgmax>(s, 2, nbands, 0, ga, as_stream(stream));
    }
    if (fmt == ASDSL_B200_FMT_Q4_128) {
        if (int rc = check_k128(K, "gemv_argmax")) return rc;
        const long long ng = K / 128;
        s[0] = StreamIn{w0, 4 * ng * 66, static_cast<long long>(M) * ng * 66};
        ga = base_args(M, K, 128);
        finish(ga);
        return launch_stream_gemv<kFmtQ4_128, kProA8, kEpiArgmax>(s, 1, nbands, 0, ga, as_stream(stream),
                                                                  rows_opt(ng * 66));
    }
    if (fmt == ASDSL_B200_FMT_Q4_128_BANDED) {
        if (!w1) return set_error(kEinval, "gemv_argmax: null pointer");
        if (int rc = check_k128(K, "gemv_argmax")) return rc;
        q128b_streams(s, w0, w1, M, K);
        ga = base_args(M, K, 128);
        finish(ga);
        return launch_stream_gemv<kFmtQ128B, kProA8, kEpiArgmax>(s, 2, nbands, 0, ga, as_stream(stream));
    }
    return set_error(kEinval, "gemv_argmax: unsupported weight format");
}
}  // namespace

extern "C" {

int asdsl_b200_gemv_argmax(int fmt, const uint8_t* w0, const uint8_t* w1, const float* x, float* y, float* out_val,
                           int32_t* out_idx, int row_base, void* scratch, size_t scratch_bytes, int M, int K,
                           void* stream) {
    return gemv_argmax_impl(fmt, w0, w1, x, y, out_val, out_idx, row_base, scratch, scratch_bytes, M, K, stream,
                            nullptr);
}

int asdsl_b200_xchg_create(int world, int rank, asdsl_b200_xchg** out, void* ipc_handle) {
    if (!out || !ipc_handle) return set_error(kEinval, "xchg_create: null pointer");
    if (world < 1 || world > 64 || rank < 0 || rank >= world) return set_error(kEinval, "xchg_create: bad rank / world");
    *out = nullptr;
    auto* x = new asdsl_b200_xchg();
    x->world = world;
    x->rank = rank;
    cudaGetDevice(&x->device);
    auto fail = [&](int rc) {
        asdsl_b200_xchg_destroy(x);
        return rc;
    };
    const size_t bytes = 2ull * world * sizeof(unsigned long long);
    if (cudaMalloc(reinterpret_cast<void**>(&x->slots), bytes) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&x->epoch), sizeof(int)) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&x->peer_table), world * sizeof(void*)) != cudaSuccess)
        return fail(set_error(asdsl::kEnomem, "xchg_create: device allocation failed"));
    if (cudaMemset(x->slots, 0, bytes) != cudaSuccess || cudaMemset(x->epoch, 0, sizeof(int)) != cudaSuccess)
        return fail(set_error(kEcuda, "xchg_create: memset failed"));
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, x->slots);
    if (e != cudaSuccess) return fail(set_error(kEcuda, std::string("xchg_create: cudaIpcGetMemHandle: ") + cudaGetErrorString(e)));
    std::memcpy(ipc_handle, &h, sizeof(h));
    *out = x;
    return kOk;
}

size_t asdsl_b200_xchg_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int asdsl_b200_xchg_open(asdsl_b200_xchg* x, const void* handles) {
    if (!x || !handles) return set_error(kEinval, "xchg_open: null pointer");
    if (x->open) return kOk;
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != x->device) return set_error(kEinval, "xchg_open: call with the exchange's device current");
    unsigned long long* table[64];
    for (int r = 0; r < x->world; ++r) {
        if (r == x->rank) {
            table[r] = x->slots;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t*>(handles) + r * sizeof(h), sizeof(h));
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            return set_error(kEcuda, std::string("xchg_open: cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
        x->mapped[r] = p;
        table[r] = static_cast<unsigned long long*>(p);
    }
    ASDSL_CUDA(cudaMemcpy(x->peer_table, table, x->world * sizeof(void*), cudaMemcpyHostToDevice));
    x->open = true;
    return kOk;
}

int asdsl_b200_xchg_destroy(asdsl_b200_xchg* x) {
    if (!x) return kOk;
    for (int r = 0; r < 64; ++r)
        if (x->mapped[r]) cudaIpcCloseMemHandle(x->mapped[r]);
    if (x->slots) cudaFree(x->slots);
    if (x->epoch) cudaFree(x->epoch);
    if (x->peer_table) cudaFree(x->peer_table);
    delete x;
    return kOk;
}

int asdsl_b200_xchg_set_stamps(asdsl_b200_xchg* x, unsigned long long* stamps, int n_slots) {
    if (!x) return set_error(kEinval, "xchg_set_stamps: null exchange");
    if (stamps && (n_slots <= 0 || (n_slots & (n_slots - 1))))
        return set_error(kEinval, "xchg_set_stamps: n_slots must be a power of two");
    x->stamps = stamps;
    x->stamp_mask = stamps ? n_slots - 1 : 0;
    return kOk;
}

int asdsl_b200_gemv_argmax_xchg(int fmt, const uint8_t* w0, const uint8_t* w1, const float* x, float* y,
                                float* out_val, int32_t* out_idx, int row_base, void* scratch, size_t scratch_bytes,
                                int M, int K, asdsl_b200_xchg* xg, void* stream) {
    if (row_base < 0)
        return set_error(kEinval, "gemv_argmax_xchg: row_base must be >= 0 (the exchange packs a 24-bit index)");
    if (!xg || !xg->open) return set_error(kEinval, "gemv_argmax_xchg: exchange not opened");
    if (static_cast<long long>(row_base) + M > (1ll << 24))
        return set_error(kEinval, "gemv_argmax_xchg: global row indices must stay below 2^24");
    return gemv_argmax_impl(fmt, w0, w1, x, y, out_val, out_idx, row_base, scratch, scratch_bytes, M, K, stream, xg);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// vector exchange: the all-reduce of the K-split down projection (row-sharded MLP).  Every rank
// holds a buffer of [2 parities][world][stride] 64-bit words, mapped into every peer over CUDA
// IPC.  A word is one float of a rank's partial in its low half and the step number in its high
// half, stored with one 64-bit relaxed system-scope store: a reader that sees the step number
// sees the float, so no fence and no separate flag are needed.  One kernel per step: CTA d
// stores this rank's partial into rank d's buffer (NVLink peer stores), then sums its slice of
// the world's partials in rank order from its own buffer, polling -- bounded -- each word until
// it carries this step's number; every rank ends with the same bits.  Buffers alternate by step
// parity: a rank stores step e + 2 only after it has seen every rank's step e + 1 words, which
// each rank stores only after its step-e kernel (and so its reads of step e) completed.
// No multicast, no library kernel on peer memory.
// ---------------------------------------------------------------------------
struct asdsl_b200_vxchg {
    int world = 1, rank = 0, device = 0, n_max = 0, stride = 0;
    unsigned long long* buf = nullptr;  // this rank's [2][world][stride] words
    // device control block: [0] last completed step, [1] CTA arrival counter, [2] stamp slot
    // mask, [4..5] the stamp buffer's address (0 = off) -- read by every launch, so that the
    // stamps reach steps replayed from CUDA graphs captured before they were turned on
    int* epoch = nullptr;
    unsigned long long** peer_buf = nullptr;  // device array [world]: every rank's buffer, mapped here
    void* mapped_buf[64] = {};
    bool open = false;
};

namespace {
constexpr int kVxThreads = 256;
constexpr int kVxMaxWorld = 16;
constexpr int kVxPerThread = 2;  // elements per thread: all their words are loaded before any wait

// grid: enough CTAs that every thread owns at most kVxPerThread elements of the vector
inline int vx_grid(int n) { return std::max(1, (n + kVxThreads * kVxPerThread - 1) / (kVxThreads * kVxPerThread)); }

// `out` may equal `add` (element i is read and written by the same thread)
__global__ void __launch_bounds__(kVxThreads)
    k_allreduce_peer(const float* __restrict__ part, float* out, const float* add, int n,
                     int stride, int world, int rank, unsigned long long* const* __restrict__ peer_buf,
                     const unsigned long long* self_buf, int* epoch, unsigned int* status) {
    // launched as a programmatic dependent of the GEMV that produced `part`: wait for it, then
    // let the next kernel launch (its weight streaming overlaps this exchange)
    grid_dependency_wait();
    grid_launch_dependents();
    const int e = epoch[0] + 1;
    const int par = e & 1;
    const unsigned long long tag = static_cast<unsigned long long>(static_cast<unsigned int>(e)) << 32;
    // stamps (CTA 0): kernel start, own slice stored to every rank, slice gathered and summed, end
    unsigned long long* stamps = reinterpret_cast<unsigned long long*>(*reinterpret_cast<const unsigned long long*>(epoch + 4));
    unsigned long long* stamp =
        (stamps && blockIdx.x == 0 && threadIdx.x == 0) ? stamps + (e & epoch[2]) * 4 : nullptr;
    if (stamp) stamp[0] = globaltimer_ns();
    // this thread's elements: i = blockIdx.x * kVxThreads * kVxPerThread + j * kVxThreads + threadIdx.x
    const int ib = blockIdx.x * kVxThreads * kVxPerThread + threadIdx.x;
    // 1. store this rank's values of those elements, tagged, into every rank's buffer
    const size_t my_off = (static_cast<size_t>(par) * world + rank) * stride;
#pragma unroll
    for (int j = 0; j < kVxPerThread; ++j) {
        const int i = ib + j * kVxThreads;
        if (i < n) {
            const unsigned long long wv = tag | __float_as_uint(part[i]);
            for (int d = 0; d < world; ++d) st_relaxed_sys_u64(peer_buf[d] + my_off + i, wv);
        }
    }
    if (stamp) stamp[1] = globaltimer_ns();
    // 2. every rank's words of those elements: all loads issued first, then a bounded wait on
    //    each word still carrying an older step, then the rank-ordered sum
    const unsigned long long* base = self_buf + static_cast<size_t>(par) * world * stride;
    unsigned long long w[kVxPerThread][kVxMaxWorld];
#pragma unroll
    for (int j = 0; j < kVxPerThread; ++j) {
        const int i = ib + j * kVxThreads;
#pragma unroll
        for (int r = 0; r < kVxMaxWorld; ++r)
            if (r < world && i < n) w[j][r] = ld_relaxed_sys_u64(base + static_cast<size_t>(r) * stride + i);
    }
    const unsigned long long t0 = globaltimer_ns();
    bool ok = true;
#pragma unroll
    for (int j = 0; j < kVxPerThread; ++j) {
        const int i = ib + j * kVxThreads;
        if (i >= n) continue;
        float acc = 0.0f;
#pragma unroll
        for (int r = 0; r < kVxMaxWorld; ++r) {
            if (r < world) {
                while (ok && (w[j][r] & 0xFFFFFFFF00000000ull) != tag) {
                    if (globaltimer_ns() - t0 > kWaitLimitNs) {
                        atomicOr(status, kStatusXchgWait);
                        ok = false;
                    } else {
                        w[j][r] = ld_relaxed_sys_u64(base + static_cast<size_t>(r) * stride + i);
                    }
                }
                const float v = __uint_as_float(static_cast<unsigned int>(w[j][r]));
                acc = (r == 0) ? v : __fadd_rn(acc, v);
            }
        }
        if (ok) out[i] = add ? __fadd_rn(acc, add[i]) : acc;
    }
    // 3. the last CTA to arrive advances the step counter (the next launch reads it)
    __syncthreads();
    if (threadIdx.x == 0) {
        if (stamp) stamp[2] = globaltimer_ns();
        const bool last = atomicAdd(epoch + 1, 1) == static_cast<int>(gridDim.x) - 1;
        if (last) {
            epoch[1] = 0;
            epoch[0] = e;
        }
        if (stamp) stamp[3] = globaltimer_ns();
    }
}
}  // namespace

extern "C" {

size_t asdsl_b200_vxchg_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int asdsl_b200_vxchg_create(int world, int rank, int n_max, asdsl_b200_vxchg** out, void* ipc_handle) {
    if (!out || !ipc_handle) return set_error(kEinval, "vxchg_create: null pointer");
    if (world < 1 || world > kVxMaxWorld || rank < 0 || rank >= world)
        return set_error(kEinval, "vxchg_create: world must be in [1, 16], rank in [0, world)");
    if (n_max <= 0 || n_max > (1 << 24)) return set_error(kEinval, "vxchg_create: vector length must be in [1, 2^24]");
    *out = nullptr;
    auto* x = new asdsl_b200_vxchg();
    x->world = world;
    x->rank = rank;
    x->n_max = n_max;
    x->stride = (n_max + 1) & ~1;  // 16-byte aligned slots
    cudaGetDevice(&x->device);
    auto fail = [&](int rc) {
        asdsl_b200_vxchg_destroy(x);
        return rc;
    };
    const size_t bbytes = 2ull * world * x->stride * sizeof(unsigned long long);
    if (cudaMalloc(reinterpret_cast<void**>(&x->buf), bbytes) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&x->epoch), 8 * sizeof(int)) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&x->peer_buf), world * sizeof(void*)) != cudaSuccess)
        return fail(set_error(asdsl::kEnomem, "vxchg_create: device allocation failed"));
    // step tags start at 1: a zeroed word never matches
    if (cudaMemset(x->buf, 0, bbytes) != cudaSuccess || cudaMemset(x->epoch, 0, 8 * sizeof(int)) != cudaSuccess)
        return fail(set_error(kEcuda, "vxchg_create: memset failed"));
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, x->buf);
    if (e != cudaSuccess)
        return fail(set_error(kEcuda, std::string("vxchg_create: cudaIpcGetMemHandle: ") + cudaGetErrorString(e)));
    std::memcpy(ipc_handle, &h, sizeof(h));
    *out = x;
    return kOk;
}

int asdsl_b200_vxchg_open(asdsl_b200_vxchg* x, const void* handles) {
    if (!x || !handles) return set_error(kEinval, "vxchg_open: null pointer");
    if (x->open) return kOk;
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != x->device) return set_error(kEinval, "vxchg_open: call with the exchange's device current");
    unsigned long long* bt[kVxMaxWorld];
    for (int r = 0; r < x->world; ++r) {
        if (r == x->rank) {
            bt[r] = x->buf;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t*>(handles) + r * sizeof(h), sizeof(h));
        const cudaError_t e = cudaIpcOpenMemHandle(&x->mapped_buf[r], h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            return set_error(kEcuda, std::string("vxchg_open: cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
        bt[r] = static_cast<unsigned long long*>(x->mapped_buf[r]);
    }
    ASDSL_CUDA(cudaMemcpy(x->peer_buf, bt, x->world * sizeof(void*), cudaMemcpyHostToDevice));
    x->open = true;
    return kOk;
}

int asdsl_b200_vxchg_destroy(asdsl_b200_vxchg* x) {
    if (!x) return kOk;
    for (int r = 0; r < 64; ++r)
        if (x->mapped_buf[r]) cudaIpcCloseMemHandle(x->mapped_buf[r]);
    if (x->buf) cudaFree(x->buf);
    if (x->epoch) cudaFree(x->epoch);
    if (x->peer_buf) cudaFree(x->peer_buf);
    delete x;
    return kOk;
}

int asdsl_b200_vxchg_set_stamps(asdsl_b200_vxchg* x, unsigned long long* stamps, int n_slots) {
    if (!x) return set_error(kEinval, "vxchg_set_stamps: null exchange");
    if (stamps && (n_slots <= 0 || (n_slots & (n_slots - 1))))
        return set_error(kEinval, "vxchg_set_stamps: n_slots must be a power of two");
    int ctl[6] = {0, 0, stamps ? n_slots - 1 : 0, 0, 0, 0};
    const unsigned long long addr = reinterpret_cast<unsigned long long>(stamps);
    std::memcpy(&ctl[4], &addr, sizeof(addr));
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != x->device) cudaSetDevice(x->device);
    const cudaError_t e = cudaMemcpy(x->epoch + 2, ctl + 2, 4 * sizeof(int), cudaMemcpyHostToDevice);
    if (prev >= 0 && prev != x->device) cudaSetDevice(prev);
    if (e != cudaSuccess) return set_error(kEcuda, std::string("vxchg_set_stamps: ") + cudaGetErrorString(e));
    return kOk;
}

int asdsl_b200_allreduce_peer(asdsl_b200_vxchg* x, const float* part, float* out, const float* add, int n,
                              void* stream) {
    if (!x || !x->open) return set_error(kEinval, "allreduce_peer: exchange not opened");
    if (!part || !out) return set_error(kEinval, "allreduce_peer: null pointer");
    if (n < 0 || n > x->n_max) return set_error(kEinval, "allreduce_peer: n exceeds the exchange's vector length");
    const uintptr_t p0 = reinterpret_cast<uintptr_t>(part), o0 = reinterpret_cast<uintptr_t>(out);
    const uintptr_t nb = static_cast<uintptr_t>(n) * sizeof(float);
    if (n > 0 && p0 < o0 + nb && o0 < p0 + nb)
        return set_error(kEinval, "allreduce_peer: the partial and the output must not overlap");
    unsigned int* st = device_status_ptr();
    if (!st) return set_error(kEcuda, "cannot resolve the device status word");
    // n == 0 still runs the step, so that every rank takes the same number of steps
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(vx_grid(n));
    cfg.blockDim = dim3(kVxThreads);
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr[1];
    if (launch_policy().pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    ASDSL_CUDA(cudaLaunchKernelEx(&cfg, k_allreduce_peer, part, out, add, n, x->stride, x->world, x->rank,
                                  static_cast<unsigned long long* const*>(x->peer_buf),
                                  static_cast<const unsigned long long*>(x->buf), x->epoch, st));
    return kOk;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// self-test of the bounded waits: a wait that nothing ever completes must give up, set its
// status bit and return, leaving the context usable
// ---------------------------------------------------------------------------
namespace {
__global__ void k_selftest_wait(int which, const unsigned long long* never_set, unsigned int* status) {
    if (threadIdx.x != 0) return;
    if (which == 0) {
        // an mbarrier expecting one arrival that never comes (the streaming pipeline's wait)
        __shared__ __align__(8) uint64_t bar;
        mbar_init(&bar, 1);
        fence_mbar_init();
        if (!mbar_wait(&bar, 0)) atomicOr(status, kStatusWaitFull);
    } else {
        // a peer word that never arrives (the cross-GPU exchange's wait)
        const unsigned long long t0 = globaltimer_ns();
        while ((ld_acquire_sys_u64(never_set) >> 56) != 1ull) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                atomicOr(status, kStatusXchgWait);
                break;
            }
        }
    }
}
}  // namespace

extern "C" {

int asdsl_b200_selftest_bounded_wait(int which, void* stream) {
    if (which != 0 && which != 1) return set_error(kEinval, "selftest_bounded_wait: which must be 0 or 1");
    unsigned int* st = device_status_ptr();
    if (!st) return set_error(kEcuda, "cannot resolve the device status word");
    unsigned long long* flag = nullptr;
    ASDSL_CUDA(cudaMalloc(reinterpret_cast<void**>(&flag), sizeof(unsigned long long)));
    cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(unsigned long long), as_stream(stream));
    if (e == cudaSuccess) {
        k_selftest_wait<<<1, 32, 0, as_stream(stream)>>>(which, flag, st);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(as_stream(stream));
    cudaFree(flag);
    ASDSL_CUDA(e);
    unsigned int v = 0;
    ASDSL_CUDA(cudaMemcpy(&v, st, sizeof(v), cudaMemcpyDeviceToHost));
    const unsigned int expect = which == 0 ? kStatusWaitFull : kStatusXchgWait;
    if (v & expect) return set_error(kEtimeout, "selftest_bounded_wait: the wait gave up as designed");
    return set_error(kEcuda, "selftest_bounded_wait: the wait did not report its timeout");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// multi-token W4A8 GEMV: one pass streams the weights once for up to 16 activation rows
// ---------------------------------------------------------------------------
// Activation scratch of the multi-token GEMVs: the tokens of one pass are quantized once into a
// slot (at most half the shared-memory budget, the per-pass limit) by k_quant_tokens.  A static
// device array (no allocation, so captured graphs need no warm-up call) of kTokSlots slots per
// device.  Each stream keeps one slot: the calls of one stream are ordered (k_quant_tokens waits
// for the previous kernel of its stream before it writes), and the first kTokSlots streams that
// call on a device get distinct slots.  Later streams share slots (assigned in turn), so
// multi-token calls on more than kTokSlots streams of one device must not overlap.
constexpr int kTokSlots = 8;
// a slot holds the A8 areas of one pass; the pipeline keeps the rest of the shared-memory budget,
// at least kMtMinRing bytes (two 20 KB stages at K = 8192), so 16 tokens of K = 8192 take one pass
constexpr size_t kMtMinRing = 40 * 1024;
constexpr size_t kTokSlotBytes = kSmemBudget - kBarBytes - kMtMinRing;
static __device__ __align__(128) unsigned char g_tok_scratch[kTokSlots * kTokSlotBytes];

namespace {
int token_scratch_slot(cudaStream_t st, uint8_t** out) {
    static std::mutex mu;
    static void* base[64] = {nullptr};
    static unsigned next[64] = {0};
    static std::vector<std::pair<cudaStream_t, unsigned>> owner[64];  // stream -> slot
    int dev = 0;
    ASDSL_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(kEinval, "gemv_multi: device index out of range");
    std::lock_guard<std::mutex> lk(mu);
    if (!base[dev]) ASDSL_CUDA(cudaGetSymbolAddress(&base[dev], g_tok_scratch));
    unsigned slot = 0;
    bool found = false;
    for (const auto& o : owner[dev])
        if (o.first == st) {
            slot = o.second;
            found = true;
            break;
        }
    if (!found) {
        slot = next[dev]++ % kTokSlots;
        owner[dev].emplace_back(st, slot);
        if (owner[dev].size() > 4096) owner[dev].erase(owner[dev].begin());  // bounded table
    }
    *out = static_cast<uint8_t*>(base[dev]) + slot * kTokSlotBytes;
    return kOk;
}

// quantize the T tokens of a pass into a scratch slot (PDL: overlaps the previous kernel's tail)
template <int PRO>
int quant_tokens(GemvArgs& ga, int T, cudaStream_t st) {
    const uint32_t xa_stride = xarea_layout_bytes(ga.K, ga.gs, false);
    if (static_cast<size_t>(xa_stride) * T > kTokSlotBytes) return set_error(kEinval, "internal: token scratch too small");
    uint8_t* slot = nullptr;
    if (int rc = token_scratch_slot(st, &slot)) return rc;
    GemvArgs g = ga;
    g.n_tokens = T;
    void* args[] = {&g, &slot, const_cast<uint32_t*>(&xa_stride)};
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(static_cast<unsigned>(T));
    cfg.blockDim = dim3(kConsumerThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (launch_policy().pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    ASDSL_CUDA(cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(&k_quant_tokens<PRO>), args));
    ga.xa_pre = slot;
    return kOk;
}

template <int FMT, int PRO>
int multi_pass(int T, const StreamIn* s, int ns, long long nb, GemvArgs ga, cudaStream_t st, const LaunchOpts& o) {
    ga.n_tokens = T;
    // from 4 rows the tokens are quantized once up front (in every CTA's prologue they cost more
    // than the extra launch); 2 rows stay in the prologue
    if (T >= 4)
        if (int rc = quant_tokens<PRO>(ga, T, st)) return rc;
    if (T <= 2) return launch_stream_gemv<FMT, PRO, kEpiStore, 2>(s, ns, nb, 0, ga, st, o);
    if (T <= 4) return launch_stream_gemv<FMT, PRO, kEpiStore, 4>(s, ns, nb, 0, ga, st, o);
    if constexpr (MmaFmt<FMT>::kSupported) {
        // 16 x 8 x 32 group dots on the tensor cores, when selected (asdsl_b200_set_mma_min_tokens);
        // off by default: on B200 the lane-dot path measures faster for 8 and 16 rows
        const int mt = launch_policy().mma_min_tokens;
        if (mt > 0 && T >= mt && T >= 5 && mma_plan_fits(s, ns, ga.K, ga.gs, T)) {
            if (T <= 8) return launch_stream_gemv_mma<FMT, PRO, 8>(s, ns, nb, ga, st, o);
            return launch_stream_gemv_mma<FMT, PRO, 16>(s, ns, nb, ga, st, o);
        }
    }
    if (T <= 8) return launch_stream_gemv<FMT, PRO, kEpiStore, 8>(s, ns, nb, 0, ga, st, o);
    return launch_stream_gemv<FMT, PRO, kEpiStore, 16>(s, ns, nb, 0, ga, st, o);
}
}  // namespace

extern "C" {

int asdsl_b200_gemv_multi(int fmt, const uint8_t* w0, const uint8_t* w1, const float* X, float* Y, int M, int K,
                          int n_tokens, void* stream) {
    if (!w0 || !X || !Y) return set_error(kEinval, "gemv_multi: null pointer");
    if (M <= 0 || K <= 0 || n_tokens <= 0) return set_error(kEinval, "gemv_multi: invalid dimensions");
    StreamIn s[2];
    int ns = 1;
    LaunchOpts o;
    int gs = 32;
    const bool q4k = (fmt == ASDSL_B200_FMT_Q4K);
    if (fmt == ASDSL_B200_FMT_PREQ) {
        if (int rc = check_k(K, 32, "gemv_multi")) return rc;
        const long long ng = K / 32;
        s[0] = StreamIn{w0, 4 * ng * 20, static_cast<long long>(M) * ng * 20};
        o = rows_opt(ng * 20);
    } else if (fmt == ASDSL_B200_FMT_PREQ2) {
        if (!w1) return set_error(kEinval, "gemv_multi: null pointer");
        if (int rc = check_k(K, 32, "gemv_multi")) return rc;
        preq2_streams(s, w0, w1, M, K);
        ns = 2;
    } else if (fmt == ASDSL_B200_FMT_Q4_128_BANDED) {
        if (!w1) return set_error(kEinval, "gemv_multi: null pointer");
        if (int rc = check_k128(K, "gemv_multi")) return rc;
        q128b_streams(s, w0, w1, M, K);
        ns = 2;
        gs = 128;
    } else if (q4k) {
        if (K % 256) return set_error(kEinval, "in_features must be divisible by 256 for Q4_K_M");
        if (K > kMaxK) return set_error(kEinval, "gemv_multi: in_features too large");
        const long long nb = K / 256;
        s[0] = StreamIn{w0, 4 * nb * 144, static_cast<long long>(M) * nb * 144};
        o = rows_opt(nb * 144);
    } else {
        return set_error(kEinval, "gemv_multi: unsupported weight format");
    }
    // tokens per pass: 16 at most, and their A8 areas within a token-scratch slot (the pipeline
    // keeps the rest of the shared memory)
    const uint32_t xa = xarea_layout_bytes(K, gs, false);
    int per_pass = static_cast<int>(kTokSlotBytes / xa);
    if (per_pass > 16) per_pass = 16;
    if (per_pass < 1) per_pass = 1;
    const long long nb = (static_cast<long long>(M) + 3) / 4;
    for (int t0 = 0; t0 < n_tokens; t0 += per_pass) {
        const int T = (n_tokens - t0 < per_pass) ? n_tokens - t0 : per_pass;
        GemvArgs ga = base_args(M, K, gs);
        ga.x = X + static_cast<long long>(t0) * K;
        ga.y = Y + static_cast<long long>(t0) * M;
        int rc = kOk;
        if (T == 1) {
            if (fmt == ASDSL_B200_FMT_PREQ) rc = launch_stream_gemv<kFmtPreq, kProA8, kEpiStore>(s, ns, nb, 0, ga, as_stream(stream), o);
            else if (fmt == ASDSL_B200_FMT_PREQ2) rc = launch_stream_gemv<kFmtPreq2, kProA8, kEpiStore>(s, ns, nb, 0, ga, as_stream(stream), o);
            else if (q4k) rc = launch_stream_gemv<kFmtQ4K, kProQ4K, kEpiStore>(s, ns, nb, 0, ga, as_stream(stream), o);
            else rc = launch_stream_gemv<kFmtQ128B, kProA8, kEpiStore>(s, ns, nb, 0, ga, as_stream(stream), o);
        } else {
            if (fmt == ASDSL_B200_FMT_PREQ) rc = multi_pass<kFmtPreq, kProA8>(T, s, ns, nb, ga, as_stream(stream), o);
            else if (fmt == ASDSL_B200_FMT_PREQ2) rc = multi_pass<kFmtPreq2, kProA8>(T, s, ns, nb, ga, as_stream(stream), o);
            else if (q4k) rc = multi_pass<kFmtQ4K, kProQ4K>(T, s, ns, nb, ga, as_stream(stream), o);
            else rc = multi_pass<kFmtQ128B, kProA8>(T, s, ns, nb, ga, as_stream(stream), o);
        }
        if (rc) return rc;
    }
    return kOk;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// allocation-free variant of gemv_argmax: the argmax scratch lives in a
// file-scope device array (one copy per device), sized for grids of up to
// kStaticArgmaxCtas CTAs: a 256-byte counter slot + 4-byte value and index per CTA.
// ---------------------------------------------------------------------------
namespace {
constexpr int kStaticArgmaxCtas = 1024;
constexpr size_t kStaticArgmaxBytes = 256 + 2 * 4 * static_cast<size_t>(kStaticArgmaxCtas);  // 8448 bytes
constexpr int kStaticMaxDevices = 64;
std::mutex g_static_scratch_mu;
void* g_static_scratch_ptr[kStaticMaxDevices] = {};
}  // namespace

static __device__ __align__(256) unsigned char g_argmax_static_scratch[kStaticArgmaxBytes];

extern "C" {

int asdsl_b200_gemv_argmax_static(int fmt, const uint8_t* w0, const uint8_t* w1, const float* x, float* y,
                                  float* out_val, int32_t* out_idx, int row_base, int M, int K, void* stream) {
    const long long max_ctas = static_cast<long long>(sm_count()) * launch_policy().ctas_per_sm;
    const size_t need = 256 + 2 * 4 * static_cast<size_t>(max_ctas);
    if (need > kStaticArgmaxBytes || asdsl_b200_argmax_scratch_bytes() > kStaticArgmaxBytes)
        return set_error(kErange, "gemv_argmax_static: this device needs " + std::to_string(need) +
                                      " bytes of argmax scratch (" + std::to_string(max_ctas) +
                                      " CTAs); the static maximum is " + std::to_string(kStaticArgmaxBytes) +
                                      " bytes (" + std::to_string(kStaticArgmaxCtas) + " CTAs)");
    int dev = 0;
    ASDSL_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kStaticMaxDevices)
        return set_error(kErange, "gemv_argmax_static: device ordinal " + std::to_string(dev) + " beyond " +
                                      std::to_string(kStaticMaxDevices - 1));
    void* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_static_scratch_mu);
        if (!g_static_scratch_ptr[dev]) {
            // first call on this device: resolve the array's address (device `dev` is current)
            // and zero it on the caller's stream; the kernel re-arms the counter after each use
            void* p = nullptr;
            ASDSL_CUDA(cudaGetSymbolAddress(&p, g_argmax_static_scratch));
            ASDSL_CUDA(cudaMemsetAsync(p, 0, kStaticArgmaxBytes, as_stream(stream)));
            g_static_scratch_ptr[dev] = p;
        }
        scratch = g_static_scratch_ptr[dev];
    }
    return asdsl_b200_gemv_argmax(fmt, w0, w1, x, y, out_val, out_idx, row_base, scratch, kStaticArgmaxBytes, M, K,
                                  stream);
}

int asdsl_b200_gateup_silu(int fmt, const uint8_t* w0, const uint8_t* w1, const float* x, float* h, int I, int K,
                           void* stream) {
    if (!w0 || !x || !h) return set_error(kEinval, "gateup_silu: null pointer");
    if (I <= 0) return set_error(kEinval, "gateup_silu: invalid dimensions");
    if (I % 4) return set_error(kEinval, "gateup_silu: intermediate size must be a multiple of 4");
    GemvArgs ga;
    StreamIn s[2];
    const long long nb = I / 4;
    if (fmt == ASDSL_B200_FMT_PREQ2) {
        if (!w1) return set_error(kEinval, "gateup_silu: null pointer");
        if (int rc = check_k(K, 32, "gateup_silu")) return rc;
        preq2_streams(s, w0, w1, 2LL * I, K);
        ga = base_args(I, K, 32);
        ga.x = x;
        ga.h = h;
        return launch_stream_gemv<kFmtPreq2, kProA8, kEpiSilu>(s, 2, nb, nb, ga, as_stream(stream));
    }
    if (fmt == ASDSL_B200_FMT_Q4_128) {
        if (int rc = check_k128(K, "gateup_silu")) return rc;
        const long long ng = K / 128;
        s[0] = StreamIn{w0, 4 * ng * 66, 2LL * I * ng * 66};
        ga = base_args(I, K, 128);
        ga.x = x;
        ga.h = h;
        return launch_stream_gemv<kFmtQ4_128, kProA8, kEpiSilu>(s, 1, nb, nb, ga, as_stream(stream), rows_opt(ng * 66));
    }
    if (fmt == ASDSL_B200_FMT_Q4_128_BANDED) {
        if (!w1) return set_error(kEinval, "gateup_silu: null pointer");
        if (int rc = check_k128(K, "gateup_silu")) return rc;
        q128b_streams(s, w0, w1, 2LL * I, K);
        ga = base_args(I, K, 128);
        ga.x = x;
        ga.h = h;
        return launch_stream_gemv<kFmtQ128B, kProA8, kEpiSilu>(s, 2, nb, nb, ga, as_stream(stream));
    }
    return set_error(kEinval, "gateup_silu: unsupported weight format");
}

// ---------------------------------------------------------------------------
// device-side weight preparation (weight_prep.cuh)
// ---------------------------------------------------------------------------
namespace {
inline bool aligned_to(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }
inline unsigned grid_for(long long items, int threads) { return static_cast<unsigned>((items + threads - 1) / threads); }
}  // namespace

int asdsl_b200_quantize_weights(const float* w, long long numel, int bits, int group_size, int symmetric,
                                int optimize_clips, uint8_t* packed, uint16_t* scales, uint16_t* zeros, void* stream) {
    if (bits != 4) return set_error(kEinval, "quantize_weights: unsupported bit-width " + std::to_string(bits));
    if (group_size != 32 && group_size != 64 && group_size != 128)
        return set_error(kEinval, "quantize_weights: group_size must be 32, 64 or 128");
    if (numel <= 0) return set_error(kEinval, "quantize_weights: empty tensor");
    if (!w || !packed || !scales || (!symmetric && !zeros)) return set_error(kEinval, "quantize_weights: null pointer");
    if (!aligned_to(w, 4) || !aligned_to(packed, 4) || !aligned_to(scales, 2) || (zeros && !aligned_to(zeros, 2)))
        return set_error(kEinval, "quantize_weights: misaligned buffer");
    const long long n_groups = (numel + group_size - 1) / group_size;
    if (n_groups > (1ll << 36)) return set_error(kEinval, "quantize_weights: tensor too large");
    constexpr int kThr = 128;
    const unsigned grid = grid_for(n_groups, kThr);
    cudaStream_t st = as_stream(stream);
    auto go = [&](auto kern) {
        kern<<<grid, kThr, 0, st>>>(w, numel, n_groups, packed, scales, symmetric ? nullptr : zeros);
    };
    const bool sym = symmetric != 0, opt = optimize_clips != 0;
    switch (group_size) {
        case 32:
            sym ? (opt ? go(k_quantize_groups<32, true, true>) : go(k_quantize_groups<32, true, false>))
                : (opt ? go(k_quantize_groups<32, false, true>) : go(k_quantize_groups<32, false, false>));
            break;
        case 64:
            sym ? (opt ? go(k_quantize_groups<64, true, true>) : go(k_quantize_groups<64, true, false>))
                : (opt ? go(k_quantize_groups<64, false, true>) : go(k_quantize_groups<64, false, false>));
            break;
        default:
            sym ? (opt ? go(k_quantize_groups<128, true, true>) : go(k_quantize_groups<128, true, false>))
                : (opt ? go(k_quantize_groups<128, false, true>) : go(k_quantize_groups<128, false, false>));
            break;
    }
    ASDSL_CUDA(cudaGetLastError());
    return kOk;
}

int asdsl_b200_repack_preq2(const uint8_t* packed, const uint16_t* scales, const uint16_t* zeros, int rows, int cols,
                            uint8_t* meta, uint8_t* quant, void* stream) {
    if (!packed || !scales || !meta || !quant) return set_error(kEinval, "repack_preq2: null pointer");
    if (int rc = check_k(cols, 32, "repack_preq2")) return rc;
    if (rows <= 0) return set_error(kEinval, "repack_preq2: invalid dimensions");
    if (!aligned_to(packed, 16) || !aligned_to(quant, 16) || !aligned_to(meta, 4) || !aligned_to(scales, 2) ||
        (zeros && !aligned_to(zeros, 2)))
        return set_error(kEinval, "repack_preq2: misaligned buffer");
    const long long work = (static_cast<long long>(rows) + 3) / 4 * 4 * (cols / 32);
    k_pack_preq2<<<grid_for(work, 256), 256, 0, as_stream(stream)>>>(packed, scales, zeros, rows, cols, meta, quant);
    ASDSL_CUDA(cudaGetLastError());
    return kOk;
}

int asdsl_b200_repack_q4_128_f32(const float* w, int rows, int cols, uint8_t* blocks, void* stream) {
    if (!w || !blocks) return set_error(kEinval, "repack_q4_128: null pointer");
    if (int rc = check_k128(cols, "repack_q4_128")) return rc;
    if (rows <= 0) return set_error(kEinval, "repack_q4_128: invalid dimensions");
    if (!aligned_to(w, 4) || !aligned_to(blocks, 2)) return set_error(kEinval, "repack_q4_128: misaligned buffer");
    const long long work = static_cast<long long>(rows) * (cols / 128);
    // one warp per group, at most 32 resident CTAs of 4 warps per SM (grid-stride beyond)
    const unsigned blocks_n = static_cast<unsigned>(std::min<long long>(grid_for(work, 4), sm_count() * 32ll));
    k_q4_128_from_f32<<<blocks_n, 128, 0, as_stream(stream)>>>(w, rows, cols, blocks);
    ASDSL_CUDA(cudaGetLastError());
    return kOk;
}

int asdsl_b200_requant_q4_128(const uint8_t* packed, const uint16_t* scales, const uint16_t* zeros, int rows, int cols,
                              uint8_t* blocks, void* stream) {
    if (!packed || !scales || !blocks) return set_error(kEinval, "requant_q4_128: null pointer");
    if (int rc = check_k128(cols, "requant_q4_128")) return rc;
    if (rows <= 0) return set_error(kEinval, "requant_q4_128: invalid dimensions");
    if (!aligned_to(scales, 2) || (zeros && !aligned_to(zeros, 2)) || !aligned_to(blocks, 2))
        return set_error(kEinval, "requant_q4_128: misaligned buffer");
    const long long work = static_cast<long long>(rows) * (cols / 128);
    k_q4_128_from_quant<<<grid_for(work, 128), 128, 0, as_stream(stream)>>>(packed, scales, zeros, rows, cols,
                                                                            blocks);
    ASDSL_CUDA(cudaGetLastError());
    return kOk;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// reference-exact numerics mode: the host CPU's RSQRTSS / RCPSS / expf tables (x86_numerics.h),
// uploaded once per device
// ---------------------------------------------------------------------------
#include "x86_numerics.h"
#include "attention_exact.cuh"

namespace {
std::mutex g_exact_mu;
ExactTabs g_exact_dev[64];
bool g_exact_ready[64] = {};

int exact_tabs_device(ExactTabs* out) {
    const HostExactTables& T = host_exact_tables();
    if (!T.ok) return set_error(kEinval, "reference-exact numerics: " + T.err);
    int dev = 0;
    ASDSL_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(kErange, "reference-exact numerics: device ordinal beyond 63");
    std::lock_guard<std::mutex> lk(g_exact_mu);
    if (!g_exact_ready[dev]) {
        // expf exceptions -> open-addressing hash table with at least 4 slots per entry
        const size_t n_exc = T.exp_exc.size() / 2;
        int bits = 4;
        while ((size_t{1} << bits) < 4 * n_exc) ++bits;
        const size_t slots = size_t{1} << bits;
        const uint32_t mask = static_cast<uint32_t>(slots - 1);
        const int shift = 32 - bits;
        const size_t n = kRcpTabSize + kRsqrtTabSize + 2 * slots;
        std::vector<uint32_t> h(n, kExpHashEmpty);
        std::memcpy(h.data(), T.rcp, 4 * kRcpTabSize);
        std::memcpy(h.data() + kRcpTabSize, T.rsqrt, 4 * kRsqrtTabSize);
        uint32_t* hash = h.data() + kRcpTabSize + kRsqrtTabSize;
        for (size_t e = 0; e < n_exc; ++e) {
            const uint32_t key = T.exp_exc[2 * e];
            uint32_t i = exp_hash_slot(key, shift);
            while (hash[2 * i] != kExpHashEmpty) i = (i + 1u) & mask;
            hash[2 * i] = key;
            hash[2 * i + 1] = T.exp_exc[2 * e + 1];
        }
        uint32_t* d = nullptr;
        ASDSL_CUDA(cudaMalloc(&d, 4 * n));
        const cudaError_t ec = cudaMemcpy(d, h.data(), 4 * n, cudaMemcpyHostToDevice);
        if (ec != cudaSuccess) {
            cudaFree(d);
            return cuda_check(ec, "reference-exact numerics: table upload");
        }
        g_exact_dev[dev].rcp = d;
        g_exact_dev[dev].rsqrt = d + kRcpTabSize;
        // 8-byte aligned: the rcp and rsqrt tables are 16 KB
        g_exact_dev[dev].exp_hash = reinterpret_cast<const uint2*>(d + kRcpTabSize + kRsqrtTabSize);
        g_exact_dev[dev].exp_hash_mask = mask;
        g_exact_dev[dev].exp_hash_shift = shift;
        g_exact_dev[dev].n_exp_exc = static_cast<int>(n_exc);
        g_exact_ready[dev] = true;
    }
    *out = g_exact_dev[dev];
    return kOk;
}
}  // namespace

namespace {
__global__ void k_exact_expf(const float* __restrict__ x, float* __restrict__ y, long long n, ExactTabs t) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        y[i] = exact_expf(x[i], t);
}
}  // namespace

extern "C" {

int asdsl_b200_exact_expf(const float* x, float* y, long long n, void* stream) {
    if (!x || !y || n < 0) return set_error(kEinval, "exact_expf: invalid arguments");
    if (n == 0) return kOk;
    ExactTabs t;
    if (int rc = exact_tabs_device(&t)) return rc;
    k_exact_expf<<<sm_count() * 8, 256, 0, as_stream(stream)>>>(x, y, n, t);
    ASDSL_CUDA(cudaGetLastError());
    return kOk;
}

int asdsl_b200_exact_numerics_init(int* n_exp_exceptions) {
    ExactTabs t;
    if (int rc = exact_tabs_device(&t)) return rc;
    if (n_exp_exceptions) *n_exp_exceptions = t.n_exp_exc;
    return kOk;
}

int asdsl_b200_exact_host_tables(uint32_t* rcp, uint32_t* rsqrt, uint32_t* exp_exc, int exp_cap, int* n_exp) {
    const HostExactTables& T = host_exact_tables();
    if (!T.ok) return set_error(kEinval, "reference-exact numerics: " + T.err);
    const int n = static_cast<int>(T.exp_exc.size() / 2);
    if (n_exp) *n_exp = n;
    if (rcp) std::memcpy(rcp, T.rcp, 4 * kRcpTabSize);
    if (rsqrt) std::memcpy(rsqrt, T.rsqrt, 4 * kRsqrtTabSize);
    if (exp_exc) {
        if (exp_cap < n) return set_error(kEinval, "exact_host_tables: exception buffer too small");
        std::memcpy(exp_exc, T.exp_exc.data(), 8ull * n);
    }
    return kOk;
}

int asdsl_b200_gemv_preq2_fused_exact(const uint8_t* meta, const uint8_t* quant, const float* x, const float* norm_w,
                                      float eps, float* y, int M, int K, void* stream) {
    if (!meta || !quant || !x || !y) return set_error(kEinval, "gemv_preq2_fused_exact: null pointer");
    if (int rc = check_k(K, 32, "gemv_preq2_fused_exact")) return rc;
    if (M < 0) return set_error(kEinval, "gemv_preq2_fused_exact: invalid dimensions");
    GemvArgs ga = base_args(M, K, 32);
    ga.x = x;
    ga.y = y;
    if (M == 0) return kOk;
    if (!norm_w) return launch_exact_gemv<kProA8X, kEpiStore>(meta, quant, M, 0, ga, as_stream(stream));
    if (K % 8) return set_error(kEinval, "gemv_preq2_fused_exact: RMSNorm needs in_features % 8 == 0");
    if (int rc = exact_tabs_device(&ga.ex)) return rc;
    ga.norm_w = norm_w;
    ga.eps = eps;
    return launch_exact_gemv<kProRmsA8X, kEpiStore>(meta, quant, M, 0, ga, as_stream(stream));
}

int asdsl_b200_gateup_silu_exact(const uint8_t* meta, const uint8_t* quant, const float* x, const float* norm_w,
                                 float eps, float* h, int I, int K, void* stream) {
    if (!meta || !quant || !x || !h) return set_error(kEinval, "gateup_silu_exact: null pointer");
    if (I <= 0 || I % 4) return set_error(kEinval, "gateup_silu_exact: intermediate size must be a positive multiple of 4");
    if (int rc = check_k(K, 32, "gateup_silu_exact")) return rc;
    GemvArgs ga = base_args(I, K, 32);
    if (int rc = exact_tabs_device(&ga.ex)) return rc;
    ga.x = x;
    ga.h = h;
    if (!norm_w) return launch_exact_gemv<kProA8X, kEpiSiluX>(meta, quant, 2LL * I, I, ga, as_stream(stream));
    if (K % 8) return set_error(kEinval, "gateup_silu_exact: RMSNorm needs in_features % 8 == 0");
    ga.norm_w = norm_w;
    ga.eps = eps;
    return launch_exact_gemv<kProRmsA8X, kEpiSiluX>(meta, quant, 2LL * I, I, ga, as_stream(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// one layer's projection set behind a synchronous host-buffer call (asdsl_b200_layer_*): the
// H2D copy of x, the four GEMVs and the D2H copy of the three results replay as one CUDA graph
// on the object's own stream, so a call costs one graph launch and one stream synchronization
// ---------------------------------------------------------------------------
struct asdsl_b200_layer {
    const uint8_t* w[8] = {};  // qkv meta, quant; o meta, quant; gate_up quant, scales; down quant, scales
    float* x_dev = nullptr;
    float* h_dev = nullptr;
    float* out_dev = nullptr;  // [qkv_rows | hidden | hidden]
    int H = 0, QKV = 0, QD = 0, I = 0;
    int device = 0;
    cudaStream_t stream = nullptr;
    float* x_pin = nullptr;
    float* out_pin = nullptr;
    float* x_map = nullptr;    // the staging's device-side (mapped) addresses
    float* out_map = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
};

namespace {
// the layer step's host transfers as kernels reading / writing the pinned staging through its
// mapped address (UVA): in a graph, a copy-engine node of a few KB cost ~10 us each, a kernel ~1 us,
// and kernels chain with programmatic dependent launch
__global__ void k_host_in(const float* __restrict__ src, float* __restrict__ dst, int n) {
    grid_launch_dependents();  // the next GEMV's producer may stream its weights already
    const int n4 = n >> 2;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n4) reinterpret_cast<float4*>(dst)[i] = reinterpret_cast<const float4*>(src)[i];
    if (i < (n & 3)) dst[4 * n4 + i] = src[4 * n4 + i];
}

__global__ void k_host_out(const float* __restrict__ src, float* __restrict__ dst, int n) {
    grid_dependency_wait();  // the last GEMV's results are complete and visible
    const int n4 = n >> 2;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n4) reinterpret_cast<float4*>(dst)[i] = __ldcg(reinterpret_cast<const float4*>(src) + i);
    if (i < (n & 3)) dst[4 * n4 + i] = __ldcg(src + 4 * n4 + i);
}

// the device-side address of a pinned host buffer (mapped into the device's address space), or
// an error: pageable or unmapped memory is refused before any kernel could touch it
int mapped_address(const void* host, const char* fn, void** dev_addr) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, host) != cudaSuccess || at.type != cudaMemoryTypeHost ||
        at.devicePointer == nullptr) {
        cudaGetLastError();
        return set_error(kEinval, std::string(fn) + ": the host buffer must be pinned and mapped (cudaMallocHost "
                                                    "/ cudaHostAlloc / torch pin_memory)");
    }
    *dev_addr = at.devicePointer;
    return kOk;
}

int layer_enqueue(asdsl_b200_layer* L) {
    {
        const int n = L->H;
        k_host_in<<<(n / 4 + 255) / 256 + 1, 256, 0, L->stream>>>(L->x_map, L->x_dev, n);
        ASDSL_CUDA(cudaGetLastError());
    }
    float* qkv = L->out_dev;
    float* o = L->out_dev + L->QKV;
    float* y = L->out_dev + L->QKV + L->H;
    if (int rc = asdsl_b200_gemv_preq2_fused(L->w[0], L->w[1], L->x_dev, qkv, L->QKV, L->H, 32, L->stream)) return rc;
    if (int rc = asdsl_b200_gemv_preq2_fused(L->w[2], L->w[3], qkv, o, L->H, L->QD, 32, L->stream)) return rc;
    if (int rc = asdsl_b200_gateup_silu(ASDSL_B200_FMT_Q4_128_BANDED, L->w[4], L->w[5], o, L->h_dev, L->I, L->H,
                                        L->stream))
        return rc;
    if (int rc = asdsl_b200_gemv_q4_128_banded(L->w[6], L->w[7], L->h_dev, y, L->H, L->I, L->stream)) return rc;
    {
        const int n = L->QKV + 2 * L->H;
        cudaLaunchConfig_t cfg;
        std::memset(&cfg, 0, sizeof(cfg));
        cfg.gridDim = dim3((n / 4 + 255) / 256 + 1);
        cfg.blockDim = dim3(256);
        cfg.stream = L->stream;
        cudaLaunchAttribute attr[1];
        if (launch_policy().pdl) {
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
        }
        ASDSL_CUDA(cudaLaunchKernelEx(&cfg, k_host_out, static_cast<const float*>(L->out_dev), L->out_map, n));
    }
    return kOk;
}

void layer_free(asdsl_b200_layer* L) {
    if (!L) return;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(L->device);
    if (L->exec) cudaGraphExecDestroy(L->exec);
    if (L->graph) cudaGraphDestroy(L->graph);
    if (L->stream) {
        cudaStreamSynchronize(L->stream);
        cudaStreamDestroy(L->stream);
    }
    if (L->x_pin) cudaFreeHost(L->x_pin);
    if (L->out_pin) cudaFreeHost(L->out_pin);
    if (prev >= 0) cudaSetDevice(prev);
    delete L;
}
}  // namespace

extern "C" {

int asdsl_b200_layer_create(const uint8_t* qkv_meta, const uint8_t* qkv_quant, const uint8_t* o_meta,
                            const uint8_t* o_quant, const uint8_t* gu_quant, const uint8_t* gu_scales,
                            const uint8_t* dn_quant, const uint8_t* dn_scales, float* x_dev, float* h_dev,
                            float* out_dev, int hidden, int qkv_rows, int q_dim, int inter, asdsl_b200_layer** out) {
    if (!out) return set_error(kEinval, "layer_create: null handle pointer");
    *out = nullptr;
    if (!qkv_meta || !qkv_quant || !o_meta || !o_quant || !gu_quant || !gu_scales || !dn_quant || !dn_scales ||
        !x_dev || !h_dev || !out_dev)
        return set_error(kEinval, "layer_create: null pointer");
    if (hidden <= 0 || qkv_rows <= 0 || q_dim <= 0 || inter <= 0 || q_dim > qkv_rows)
        return set_error(kEinval, "layer_create: invalid dimensions");
    if ((reinterpret_cast<uintptr_t>(x_dev) | reinterpret_cast<uintptr_t>(out_dev)) & 15u)
        return set_error(kEinval, "layer_create: x_dev and out_dev must be 16-byte aligned");
    auto* L = new asdsl_b200_layer();
    const uint8_t* w[8] = {qkv_meta, qkv_quant, o_meta, o_quant, gu_quant, gu_scales, dn_quant, dn_scales};
    for (int i = 0; i < 8; ++i) L->w[i] = w[i];
    L->x_dev = x_dev;
    L->h_dev = h_dev;
    L->out_dev = out_dev;
    L->H = hidden;
    L->QKV = qkv_rows;
    L->QD = q_dim;
    L->I = inter;
    auto fail = [&](int rc) {
        layer_free(L);
        return rc;
    };
    if (cudaGetDevice(&L->device) != cudaSuccess) return fail(set_error(kEcuda, "layer_create: no CUDA device"));
    if (cudaStreamCreateWithFlags(&L->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMallocHost(&L->x_pin, 4ull * hidden) != cudaSuccess ||
        cudaMallocHost(&L->out_pin, 4ull * (qkv_rows + 2ll * hidden)) != cudaSuccess)
        return fail(set_error(kEnomem, "layer_create: stream or pinned staging"));
    std::memset(L->x_pin, 0, 4ull * hidden);
    {
        void* dx = nullptr;
        void* dout = nullptr;
        if (int rc = mapped_address(L->x_pin, "layer_create", &dx)) return fail(rc);
        if (int rc = mapped_address(L->out_pin, "layer_create", &dout)) return fail(rc);
        L->x_map = static_cast<float*>(dx);
        L->out_map = static_cast<float*>(dout);
    }
    // one eager step (kernel attributes are set on first use, outside any capture), then the graph
    if (int rc = layer_enqueue(L)) return fail(rc);
    if (cudaStreamSynchronize(L->stream) != cudaSuccess) return fail(set_error(kEcuda, "layer_create: first step"));
    if (cudaStreamBeginCapture(L->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
        return fail(set_error(kEcuda, "layer_create: capture"));
    const int rc = layer_enqueue(L);
    const cudaError_t ec = cudaStreamEndCapture(L->stream, &L->graph);
    if (rc) return fail(rc);
    if (ec != cudaSuccess || cudaGraphInstantiate(&L->exec, L->graph, 0) != cudaSuccess)
        return fail(set_error(kEcuda, "layer_create: graph"));
    *out = L;
    return kOk;
}

int asdsl_b200_layer_forward(asdsl_b200_layer* L, const float* x_host, float* out_host) {
    if (!L || !x_host || !out_host) return set_error(kEinval, "layer_forward: null pointer");
    int cur = 0;
    ASDSL_CUDA(cudaGetDevice(&cur));
    if (cur != L->device) ASDSL_CUDA(cudaSetDevice(L->device));
    std::memcpy(L->x_pin, x_host, 4ull * L->H);
    cudaError_t ec = cudaGraphLaunch(L->exec, L->stream);
    if (ec == cudaSuccess) ec = cudaStreamSynchronize(L->stream);
    if (cur != L->device) cudaSetDevice(cur);
    ASDSL_CUDA(ec);
    std::memcpy(out_host, L->out_pin, 4ull * (L->QKV + 2ll * L->H));
    return kOk;
}

int asdsl_b200_layer_destroy(asdsl_b200_layer* L) {
    layer_free(L);
    return kOk;
}


int asdsl_b200_host_to_device(const float* host_pinned, float* dev, long long n, void* stream) {
    if (!host_pinned || !dev || n < 0 || n > 0x7fffffffLL) return set_error(kEinval, "host_to_device: invalid arguments");
    if (n == 0) return kOk;
    void* src = nullptr;
    if (int rc = mapped_address(host_pinned, "host_to_device", &src)) return rc;
    if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dev)) & 15u)
        return set_error(kEinval, "host_to_device: both buffers must be 16-byte aligned");
    const int ni = static_cast<int>(n);
    k_host_in<<<static_cast<unsigned>((n / 4 + 255) / 256 + 1), 256, 0, as_stream(stream)>>>(
        static_cast<const float*>(src), dev, ni);
    ASDSL_CUDA(cudaGetLastError());
    return kOk;
}

int asdsl_b200_device_to_host(const float* dev, float* host_pinned, long long n, void* stream) {
    if (!host_pinned || !dev || n < 0 || n > 0x7fffffffLL) return set_error(kEinval, "device_to_host: invalid arguments");
    if (n == 0) return kOk;
    void* dst = nullptr;
    if (int rc = mapped_address(host_pinned, "device_to_host", &dst)) return rc;
    if ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(dev)) & 15u)
        return set_error(kEinval, "device_to_host: both buffers must be 16-byte aligned");
    const int ni = static_cast<int>(n);
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(static_cast<unsigned>((n / 4 + 255) / 256 + 1));
    cfg.blockDim = dim3(256);
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr[1];
    if (launch_policy().pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    ASDSL_CUDA(cudaLaunchKernelEx(&cfg, k_host_out, dev, static_cast<float*>(dst), ni));
    return kOk;
}

}  // extern "C"

// device-resident decode engine (asdsl_b200_engine_*)
#include "engine.cuh"
