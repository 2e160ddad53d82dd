/*
 * Test infrastructure only (oracle).  An extern "C" face over the reference's
 * own compiled C++ kernels, so Python (ctypes) can call them without the
 * reference's pybind wrappers: those release the GIL before touching numpy
 * buffers and crash under pybind11 3.x (asdsl/kernels/native/gemv_q4_avx2.cpp
 * :1357, :1373, :1388, :1411, :1428).
 *
 * Nothing in the product links this file; it is built only into oracle/_ref/
 * by oracle/Makefile, next to the reference's sources compiled where they lie.
 */
#include <cstdint>
#include <cstdlib>
#include <exception>
#include <cstdio>

// The engine ops (swiglu_inplace, rmsnorm_f32, ...) are private members of UnifiedEngine that
// touch no member state; this test-only face opens them to call them on a zeroed object.
#define private public
#include "unified_engine.h"
#undef private

// Declarations of the reference's C++ entry points
// (asdsl/kernels/native/gemv_q4_kernel.h:25-121, unified_engine.h:114-137).
void quantize_activation_avx2(const float* x, int8_t* x_q8, float* x_scales, int in_features, int group_size);
void gemv_preq2_fused_avx2(const uint8_t* meta, const uint8_t* quant, const float* x_fp32, float* y,
                           int out_features, int in_features, int group_size);
void gemv_preq2_avx2(const uint8_t* meta, const uint8_t* quant, const int8_t* x_q8, const float* x_scales,
                     float* y, int out_features, int in_features, int group_size);
void gemv_q4_32_preq_avx2(const uint8_t* blocks, const int8_t* x_q8, const float* x_scales, float* y,
                          int out_features, int in_features, int group_size);
void gemv_q4_32_preq_fused_avx2(const uint8_t* blocks, const float* x_fp32, float* y,
                                int out_features, int in_features, int group_size);
void gemv_q4_128_preq_avx2(const uint8_t* blocks, const int8_t* x_q8, const float* x_scales, float* y,
                           int out_features, int in_features, int group_size);
void gemv_q4_s256_preq_avx2(const uint8_t* blocks, const int8_t* x_q8, const float* x_scales, float* y,
                            int out_features, int in_features, int group_size);
void gemv_q4km_q8_avx2(const uint8_t* weights_q4km, const float* x, float* y, int out_features, int in_features);
void gemm_q4_128_q8_avx2(const uint8_t* blocks, const float* x_batch, float* y_batch, int out_features,
                         int in_features, int group_size, int batch_size);
void gemv_q4_packed_impl_v2(const uint8_t* w_packed, const float* x, const float* scales, const float* biases,
                            float* y, int M, int K, int group_size);
void gemv_q4_unpacked_impl(const uint8_t* w, const float* x, const float* scales, const float* biases,
                           float* y, int M, int K, int group_size);
// QCSD draft bank (asdsl/kernels/native/gemv_q2_kernels.h)
void gemv_q2_packed_impl(const uint8_t* w_packed, const float* x, const float* scales, const float* biases,
                         float* y, int M, int K, int group_size);
void gemv_q2_unpacked_impl(const uint8_t* w, const float* x, const float* scales, const float* biases, float* y,
                           int M, int K, int group_size);

#define SHIM_TRY(expr)                                   \
    try {                                                \
        expr;                                            \
        return 0;                                        \
    } catch (const std::exception& e) {                  \
        std::fprintf(stderr, "ref_shim: %s\n", e.what()); \
        return 1;                                        \
    } catch (...) {                                      \
        return 2;                                        \
    }

extern "C" {

int ref_quantize_activation(const float* x, int8_t* xq, float* xs, int K, int gs) {
    SHIM_TRY(quantize_activation_avx2(x, xq, xs, K, gs));
}
int ref_gemv_preq2_fused(const uint8_t* meta, const uint8_t* quant, const float* x, float* y, int M, int K, int gs) {
    SHIM_TRY(gemv_preq2_fused_avx2(meta, quant, x, y, M, K, gs));
}
int ref_gemv_preq2(const uint8_t* meta, const uint8_t* quant, const int8_t* xq, const float* xs, float* y,
                   int M, int K, int gs) {
    SHIM_TRY(gemv_preq2_avx2(meta, quant, xq, xs, y, M, K, gs));
}
int ref_gemv_q4_32_preq(const uint8_t* blocks, const int8_t* xq, const float* xs, float* y, int M, int K, int gs) {
    SHIM_TRY(gemv_q4_32_preq_avx2(blocks, xq, xs, y, M, K, gs));
}
int ref_gemv_q4_32_preq_fused(const uint8_t* blocks, const float* x, float* y, int M, int K, int gs) {
    SHIM_TRY(gemv_q4_32_preq_fused_avx2(blocks, x, y, M, K, gs));
}
int ref_gemv_q4_128(const uint8_t* blocks, const int8_t* xq, const float* xs, float* y, int M, int K, int gs) {
    SHIM_TRY(gemv_q4_128_preq_avx2(blocks, xq, xs, y, M, K, gs));
}
int ref_gemv_q4_s256(const uint8_t* blocks, const int8_t* xq, const float* xs, float* y, int M, int K, int gs) {
    SHIM_TRY(gemv_q4_s256_preq_avx2(blocks, xq, xs, y, M, K, gs));
}
int ref_gemv_q4km(const uint8_t* w, const float* x, float* y, int M, int K) {
    SHIM_TRY(gemv_q4km_q8_avx2(w, x, y, M, K));
}
int ref_gemm_q4_128(const uint8_t* blocks, const float* x, float* y, int M, int K, int gs, int batch) {
    SHIM_TRY(gemm_q4_128_q8_avx2(blocks, x, y, M, K, gs, batch));
}
int ref_gemv_q4_packed(const uint8_t* w, const float* x, const float* s, const float* b, float* y,
                       int M, int K, int gs) {
    SHIM_TRY(gemv_q4_packed_impl_v2(w, x, s, b, y, M, K, gs));
}
int ref_gemv_q4_unpacked(const uint8_t* w, const float* x, const float* s, const float* b, float* y,
                         int M, int K, int gs) {
    SHIM_TRY(gemv_q4_unpacked_impl(w, x, s, b, y, M, K, gs));
}

int ref_gemv_q2_packed(const uint8_t* w, const float* x, const float* s, const float* b, float* y, int M, int K,
                       int gs) {
    SHIM_TRY(gemv_q2_packed_impl(w, x, s, b, y, M, K, gs));
}
int ref_gemv_q2_unpacked(const uint8_t* w, const float* x, const float* s, const float* b, float* y, int M, int K,
                         int gs) {
    SHIM_TRY(gemv_q2_unpacked_impl(w, x, s, b, y, M, K, gs));
}

namespace {
asdsl::UnifiedEngine* op_host() {
    static void* p = std::calloc(1, sizeof(asdsl::UnifiedEngine));
    return static_cast<asdsl::UnifiedEngine*>(p);
}
}  // namespace

// UnifiedEngine::swiglu_inplace (unified_engine.cpp:836-857): gate[i] = silu(gate[i]) * up[i]
int ref_swiglu(float* gate, float* up, int n) { SHIM_TRY(op_host()->swiglu_inplace(gate, up, n, 0.0f)); }
// UnifiedEngine::rmsnorm_f32 (unified_engine.cpp:499-524)
int ref_rmsnorm(float* out, const float* in, const float* w, int n, float eps) {
    SHIM_TRY(op_host()->rmsnorm_f32(out, in, w, n, eps));
}

}  // extern "C"
