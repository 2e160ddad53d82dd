/*
 * asdsl_oracle.h -- CPU restatement of the reference's W4A8 decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg may load this library, and only as the checker
 * (or the timed CPU baseline).  The product (asdsl-framework_b200/) never
 * links or calls it.
 *
 * Every function names the reference file:line it restates.  Parity of this
 * restatement is pinned against the reference itself (oracle/_ref, compiled
 * from the reference sources by oracle/Makefile) and against golden fixtures
 * generated from the reference (tests/golden/).
 */
#ifndef ASDSL_ORACLE_H
#define ASDSL_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* A8 activation quantizer, asdsl/kernels/native/gemv_q4_preq_restored.cpp:505-549 */
void or_quantize_activation(const float* x, int8_t* xq, float* xs, int32_t* xsum, int K, int gs);
/* Q4_K's own A8, asdsl/kernels/native/gemv_q4_avx2.cpp:374-402 */
void or_quantize_activation_q4k(const float* x, int8_t* xq, float* xs, int K);

/* GEMVs over pre-quantized activations */
void or_gemv_preq2_q8(const uint8_t* meta, const uint8_t* quant, const int8_t* xq, const float* xs,
                      float* y, int M, int K);                      /* gemv_preq2_avx2.cpp:196-297 */
void or_gemv_preq_q8(const uint8_t* blocks, const int8_t* xq, const float* xs, float* y, int M, int K);
                                                                    /* gemv_q4_preq_restored.cpp:305-336,338-473 */
void or_gemv_q4_128_q8(const uint8_t* blocks, const int8_t* xq, const float* xs, float* y, int M, int K);
                                                                    /* gemv_q4_128.cpp:94-257 */
int or_gemm_q4_128_f32(const uint8_t* blocks, const float* x, float* y, int M, int K, int gs, int batch);
                                                                    /* gemv_q4_128.cpp:262-306 */
void or_gemv_q4_s256_q8(const uint8_t* blocks, const int8_t* xq, const float* xs, float* y, int M, int K);
                                                                    /* gemv_q4_s256.cpp:83-209 */
/* fp32-activation entries (A8 inside, as the reference's fused entries) */
void or_gemv_preq2_fused(const uint8_t* meta, const uint8_t* quant, const float* x, float* y, int M, int K);
void or_gemv_q4km(const uint8_t* w, const float* x, float* y, int M, int K);   /* gemv_q4_avx2.cpp:357-420 */
void or_gemv_q4_packed(const uint8_t* w, const float* x, const float* scales, const float* biases,
                       float* y, int M, int K, int gs);
/* QCSD draft bank (gemv_q2_avx2.cpp:128-174, :53-118) */
void or_gemv_q2_packed(const uint8_t* w, const float* x, const float* scales, const float* biases, float* y,
                       int M, int K, int gs);
void or_gemv_q2_unpacked(const uint8_t* w, const float* x, const float* scales, const float* biases, float* y,
                         int M, int K, int gs);             /* gemv_q4_avx2.cpp:665-749 */

/* Engine-side weight quantizers (unified_engine.cpp:320-400 and :411-461) */
void or_lmhead_quant_q4_32_preq2(const uint16_t* w_f16, uint8_t* meta, uint8_t* quant, int rows, int cols);
void or_lmhead_quant_q4_128(const uint16_t* w_f16, uint8_t* blocks, int rows, int cols);

/* GCC -ffast-math's 1/sqrt(a) and 1/d on this host: RSQRTSS / RCPSS estimate + one Newton step */
float or_nr_rsqrt(float a);
float or_host_rcp(float a);   /* the host's raw RCPSS / RSQRTSS estimates */
float or_host_rsqrt(float a);
void or_expf_array(const float* x, float* y, long n);
float or_nr_recip(float d);

/* Engine ops (unified_engine.cpp) */
void or_rmsnorm(float* out, const float* in, const float* w, int n, float eps);          /* :499-524 */
void or_residual_add_rmsnorm(float* hidden, float* residual, const float* w, int n, float eps); /* :663-693 */
void or_rope(float* q, float* k, const float* cos_t, const float* sin_t, int pos, int rotary_dim,
             int n_heads, int n_kv_heads, int head_dim);                                   /* :768-801 */
void or_swiglu(float* gate, const float* up, int n);                                       /* :803-857 */
int  or_argmax(const float* v, int n);                                                     /* :207-233 */
void or_kv_write(int8_t* kq, float* ks, int8_t* vq, float* vs, const float* k, const float* v,
                 int n_kv_heads, int head_dim);                                            /* :859-920 */
void or_attention(float* out, const float* q, const int8_t* kq, const float* ks, const int8_t* vq,
                  const float* vs, int seq_pos, int n_heads, int n_kv_heads, int head_dim,
                  long pos_stride_q8, long pos_stride_sc);                                 /* :922-1027 */

/* Whole-model decode step (UnifiedEngine::forward_token, unified_engine.cpp:1339-1688,
 * C0 branch: fused preq2 GEMVs, gs=32, lm_head preq2 g32). */
typedef struct {
    int num_layers, hidden, n_heads, n_kv_heads, head_dim, inter, vocab, max_seq, rotary_dim;
    float eps;
    const uint16_t* embed_f16;        /* [vocab, hidden] */
    const float* output_norm;         /* [hidden] */
    const uint8_t* lm_meta;           /* preq2 meta of lm_head */
    const uint8_t* lm_quant;          /* preq2 quant of lm_head */
    const float* cos_t;               /* [max_seq, rotary_dim/2] */
    const float* sin_t;
    const float* const* rms_att;      /* [L][hidden] */
    const float* const* rms_ffn;
    const uint8_t* const* qkv_meta;  const uint8_t* const* qkv_quant;
    const uint8_t* const* o_meta;    const uint8_t* const* o_quant;
    const uint8_t* const* gu_meta;   const uint8_t* const* gu_quant;
    const uint8_t* const* dn_meta;   const uint8_t* const* dn_quant;
} or_model_t;

typedef struct or_engine or_engine_t;
or_engine_t* or_engine_create(const or_model_t* m);
void or_engine_destroy(or_engine_t* e);
void or_engine_reset(or_engine_t* e);
/* Returns 0 on success; logits may be NULL (prompt tokens before the last). */
int or_engine_forward_token(or_engine_t* e, int token, int pos, float* logits);

#ifdef __cplusplus
}
#endif
#endif
