/*
 * asdsl_b200.h -- C ABI of the B200-native ASDSL W4A8 decode hot path.
 *
 * Every entry point takes plain pointers and sizes.  Unless a comment says
 * otherwise, array arguments are DEVICE pointers (cudaMalloc / torch CUDA
 * storage) that are 16-byte aligned, and work is enqueued on `stream`
 * (a cudaStream_t passed as void*; NULL = the legacy default stream) without
 * synchronizing.  Functions return ASDSL_B200_OK or an error code; the message
 * of the last error on the calling thread is returned by asdsl_b200_last_error().
 *
 * Each declaration cites the reference interface it replaces
 * (aarushk09/asdsl-framework, paths relative to the repository root).
 */
#ifndef ASDSL_B200_H
#define ASDSL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes: the reference's exception classes map onto them
 * (std::invalid_argument -> EINVAL, std::out_of_range -> ERANGE) */
#define ASDSL_B200_OK 0
#define ASDSL_B200_EINVAL 1   /* bad argument (ValueError) */
#define ASDSL_B200_ERANGE 2   /* index out of range (IndexError) */
#define ASDSL_B200_ECUDA 3    /* CUDA runtime error (RuntimeError) */
#define ASDSL_B200_ENCCL 4    /* NCCL error (RuntimeError) */
#define ASDSL_B200_ETIMEOUT 5 /* a bounded device-side wait gave up */
#define ASDSL_B200_ENOMEM 6   /* device allocation failed */

/* weight formats accepted by asdsl_b200_gemv_w4a8 */
#define ASDSL_B200_FMT_PREQ2 0  /* meta [M][K/32][4] + quant [ceil(M/4)][K/32][64] (repack_preq2.py:22-46) */
#define ASDSL_B200_FMT_PREQ 1   /* [M][K/32][20] blocks (repack_q4_32.py:63-102) */
#define ASDSL_B200_FMT_Q4_128 2 /* [M][K/128][66] blocks (repack_q4_128.py:34-92) */
#define ASDSL_B200_FMT_S256 3   /* [M][K/256][144] blocks (gemv_q4_s256.cpp:1-17) */
#define ASDSL_B200_FMT_Q4_128_BANDED 4 /* device re-layout of Q4_128: quant [ceil(M/4)][K/128][4][64] +
                                          scales [ceil(M/4)][K/128][4] fp16 (asdsl_b200_relayout_q4_128) */
#define ASDSL_B200_FMT_Q4K 5    /* [M][K/256][144] reference-interpretation Q4_K (gemv_q4_avx2.cpp:110-120) */

const char* asdsl_b200_version(void);
const char* asdsl_b200_last_error(void);

/* Process-wide launch policy of the streaming GEMVs: CTAs per SM (1 or 2; 1 leaves room
 * for the next kernel of a dependent chain to start early) and programmatic dependent
 * launch (nonzero = on, the default).  No reference counterpart: the reference's CPU
 * threading knobs (ASDSL_PERSISTENT_POOL, ASDSL_CHUNKED_GEMV, engine_flags.hpp:8-15,
 * gemv_chunked.hpp:16-45) play this role there. */
int asdsl_b200_set_launch_policy(int ctas_per_sm, int use_pdl);
/* No reference counterpart.  Multi-token GEMVs (asdsl_b200_gemv_multi) with at least n_tokens rows
 * (and at least 5) compute their group dots with int8 tensor-core MMAs (mma.sync m16n8k32) instead
 * of lane dp4a chains; 0 (the default) never does.  Same results within the multi-token tolerance
 * (only the float summation order across groups differs). */
int asdsl_b200_set_mma_min_tokens(int n_tokens);

/* Reads (and with clear != 0 resets) the current device's status word: bits
 * set by kernels whose bounded waits gave up.  Synchronizes the device. */
int asdsl_b200_device_status(unsigned int* status, int clear);

/* Per-CTA timeline of the streaming GEMVs, the counterpart of the reference's ASDSL_ENGINE_PROFILE
 * stage breakdown (asdsl/kernels/native/unified_engine.cpp:74-90, :1675).  buf: device memory of
 * asdsl_b200_timeline_bytes(slots_per_block) bytes, 16-byte aligned: 1024 uint32 per-block slot
 * counters, then records [1024 blocks][slots_per_block][16 events] of 16 bytes {%globaltimer ns,
 * event | template << 4 | SM << 24, launch number}.  Every CTA takes its block's next slot and
 * writes its start (1), dependency wait (2), activation arrival (7), RMSNorm reduction (0),
 * prologue end (3), first and last chunk landed (8, 9), consumers' end (4: warp 0, 5: all) and the
 * producer's last copy (6).  buf = NULL turns it off.  Records exist only in the timeline build,
 * libasdsl_b200_timeline.so (compiled with ASDSL_B200_TIMELINE=1); the default library keeps
 * its kernels free of the hooks and returns ASDSL_B200_EINVAL for a non-NULL buf. */
int asdsl_b200_timeline_set(void* buf, unsigned int slots_per_block);
size_t asdsl_b200_timeline_bytes(unsigned int slots_per_block);

/* Self-test of the failure detection (no reference counterpart): runs one wait that nothing
 * ever completes -- which 0: an mbarrier of the streaming pipeline, 1: a cross-GPU exchange
 * word -- and returns ASDSL_B200_ETIMEOUT once the 2 s limit made it give up and set its
 * status bit (the bit stays set until asdsl_b200_device_status clears it).  Blocks ~2 s. */
int asdsl_b200_selftest_bounded_wait(int which, void* stream);

/* A8 activation quantization.
 * Replaces quantize_activation_avx2 (asdsl/kernels/native/gemv_q4_preq_restored.cpp:505-549;
 * binding asdsl/kernels/native/gemv_q4_avx2.cpp:1352-1365).
 * x[K] fp32 -> xq[K] int8, xs[K/gs] fp32; xsum[K/gs] int32 (optional, may be NULL). */
int asdsl_b200_quantize_activation(const float* x, int8_t* xq, float* xs, int32_t* xsum, int in_features,
                                   int group_size, void* stream);

/* preq2 W4A8 GEMV with fused A8 (gs 32).
 * Replaces gemv_preq2_fused_avx2 (asdsl/kernels/native/gemv_preq2_avx2.cpp:301-319;
 * binding gemv_q4_avx2.cpp:1405-1420). */
int asdsl_b200_gemv_preq2_fused(const uint8_t* meta, const uint8_t* quant, const float* x, float* y,
                                int out_features, int in_features, int group_size, void* stream);

/* preq2 W4A8 GEMV on caller-quantized activations.
 * Replaces gemv_preq2_avx2 (asdsl/kernels/native/gemv_preq2_avx2.cpp:321-337). */
int asdsl_b200_gemv_preq2(const uint8_t* meta, const uint8_t* quant, const int8_t* x_q8, const float* x_scales,
                          float* y, int out_features, int in_features, int group_size, void* stream);

/* preq (20-byte block) W4A8 GEMV on caller-quantized activations.
 * Replaces gemv_q4_32_preq_avx2 (asdsl/kernels/native/gemv_q4_preq_restored.cpp:551-577). */
int asdsl_b200_gemv_q4_32_preq(const uint8_t* blocks, const int8_t* x_q8, const float* x_scales, float* y,
                               int out_features, int in_features, int group_size, void* stream);

/* preq W4A8 GEMV with fused A8.
 * Replaces gemv_q4_32_preq_fused_avx2 / _4row / _8row / _g4fused_4row
 * (asdsl/kernels/native/gemv_q4_preq_restored.cpp:579-669). */
int asdsl_b200_gemv_q4_32_preq_fused(const uint8_t* blocks, const float* x, float* y, int out_features,
                                     int in_features, int group_size, void* stream);

/* Q4_128 symmetric W4A8 GEMV on caller-quantized activations (gs 128).
 * Replaces gemv_q4_128_preq_avx2 (asdsl/kernels/native/gemv_q4_128.cpp:94-257;
 * binding gemv_q4_avx2.cpp:1422-1437). */
int asdsl_b200_gemv_q4_128(const uint8_t* blocks, const int8_t* x_q8, const float* x_scales, float* y,
                           int out_features, int in_features, int group_size, void* stream);

/* Batched prompt GEMM on fp32 activations over Q4_128 blocks [M][K/128][66] (no A8): Y[b][M] for
 * b < min(batch, 64) of X[b][K], each row's per-group 8-lane fma dots in the reference's order, so
 * the outputs are bit-identical; Y rows b >= 64 are not written, as in the reference.
 * Replaces gemm_q4_128_q8_avx2 (asdsl/kernels/native/gemv_q4_128.cpp:262-306), the GEMM of the
 * reference engine's forward_batch for g128 projections (unified_engine.cpp:1154-1215).
 * group_size != 128 -> EINVAL (the reference's invalid_argument); blocks 2-byte and X 16-byte
 * aligned; in_features a multiple of 128. */
int asdsl_b200_gemm_q4_128_f32(const uint8_t* blocks, const float* X, float* Y, int out_features, int in_features,
                               int group_size, int batch, void* stream);

/* Q4_128 GEMV with fused A8 at gs 128: quantize_activation_avx2(..., 128) followed
 * by gemv_q4_128_preq_avx2, as the engine's C0.1 branches do
 * (asdsl/kernels/native/unified_engine.cpp:1532-1538, :1592-1598). */
int asdsl_b200_gemv_q4_128_fused(const uint8_t* blocks, const float* x, float* y, int out_features,
                                 int in_features, void* stream);

/* Q4_S256 W4A8 GEMV on caller-quantized activations (activation gs 32).
 * Replaces gemv_q4_s256_preq_avx2 (asdsl/kernels/native/gemv_q4_s256.cpp:83-209). */
int asdsl_b200_gemv_q4_s256(const uint8_t* blocks, const int8_t* x_q8, const float* x_scales, float* y,
                            int out_features, int in_features, int group_size, void* stream);

/* Q4_K (reference interpretation: fp16 d, fp16 dmin, 16 6-bit LE values, 8x16 nibble bytes)
 * GEMV with its own A8.  Replaces gemv_q4km_q8_avx2 (asdsl/kernels/native/gemv_q4_avx2.cpp:357-420;
 * binding :1318-1348). */
int asdsl_b200_gemv_q4km(const uint8_t* weights_q4km, const float* x, float* y, int out_features,
                         int in_features, void* stream);

/* fp32-activation packed W4 GEMV, `batch` independent activation rows x[batch][K] -> y[batch][M].
 * Replaces gemv_q4_packed_impl_v2 and its binding py_gemv_q4_packed
 * (asdsl/kernels/native/gemv_q4_avx2.cpp:665-749, :1084-1126). */
int asdsl_b200_gemv_q4_packed(const uint8_t* w_packed, const float* x, const float* scales, const float* biases,
                              float* y, int M, int K, int group_size, int batch, void* stream);

/* 2-bit fp32-activation GEMVs (the QCSD draft bank): y[m] = sum_g scale[m,g] * dot(codes, x_g) +
 * bias[m,g] * sum(x_g), codes 0..3.  _packed: four codes per byte (code j in bits 2j..2j+1),
 * rows of K/4 bytes; _unpacked: one code per byte.  scales / biases fp32 [M][K/gs].  K <= 32768.
 * Replace gemv_q2_packed_impl / gemv_q2_unpacked_impl (asdsl/kernels/native/gemv_q2_avx2.cpp:128-174,
 * :53-118) and their bindings gemv_q2_packed / gemv_q2_unpacked (:346-372, :300-340). */
int asdsl_b200_gemv_q2_packed(const uint8_t* w_packed, const float* x, const float* scales, const float* biases,
                              float* y, int out_features, int in_features, int group_size, void* stream);
int asdsl_b200_gemv_q2_unpacked(const uint8_t* w, const float* x, const float* scales, const float* biases,
                                float* y, int out_features, int in_features, int group_size, void* stream);

/* fp32-activation GEMV on unpacked (one code per byte) weights.
 * Replaces gemv_q4_unpacked_impl (asdsl/kernels/native/gemv_q4_avx2.cpp:755-806). */
int asdsl_b200_gemv_q4_unpacked(const uint8_t* w, const float* x, const float* scales, const float* biases,
                                float* y, int M, int K, int group_size, void* stream);

/* Batched fp32-activation packed GEMV, Y[B][M] = W x X[B][K]^T.
 * Replaces matmul_batch_q4_impl (asdsl/kernels/native/gemv_q4_avx2.cpp:950-1021). */
int asdsl_b200_matmul_batch_q4(const uint8_t* w_packed, const float* scales, const float* biases,
                               const float* X_batch, float* Y_batch, int M, int K, int B, int group_size,
                               void* stream);

/* ---- device-side weight preparation (byte-exact with the reference's NumPy pipeline) ---- */
/* quantize_weights(w, bits=4, group_size, symmetric, optimize_clips) (asdsl/quantization/core.py:358-424,
 * clip search :291-355): w fp32 [numel] on the device, padded with zeros to a multiple of group_size
 * (32, 64 or 128); packed = ceil(numel/gs)*gs/2 bytes (low nibble = even element, :555-561), scales
 * (and zeros unless symmetric, then NULL) = ceil(numel/gs) fp16 values.  bits != 4 -> EINVAL. */
int asdsl_b200_quantize_weights(const float* w, long long numel, int bits, int group_size, int symmetric,
                                int optimize_clips, uint8_t* packed, uint16_t* scales, uint16_t* zeros, void* stream);
/* gs-32 quantize_weights output -> preq2 meta + quant, i.e. repack_asymmetric_to_q4_32_blocks
 * (repack_q4_32.py:63-102; bias = -zero*scale, or -7.5*scale when zeros is NULL) followed by
 * repack_preq_blocks_to_preq2 (repack_preq2.py:22-46).  meta rows*cols/32*4 bytes, quant
 * ceil(rows/4)*(cols/32)*64 bytes (16-byte aligned), rows past `rows` in the last band zero. */
int asdsl_b200_repack_preq2(const uint8_t* packed, const uint16_t* scales, const uint16_t* zeros, int rows, int cols,
                            uint8_t* meta, uint8_t* quant, void* stream);
/* repack_fp32_to_q4_128_blocks (repack_q4_128.py:22-31, :72-92): fp32 [rows][cols] -> Q4_128 blocks
 * [rows][cols/128][66]. */
int asdsl_b200_repack_q4_128_f32(const float* w, int rows, int cols, uint8_t* blocks, void* stream);
/* The C0.1 requant (build_c01_gs128_blocks, experiments/phi4_cpu_run.py:3482-3517): a gs-32
 * quantize_weights output dequantized as q*scale + bias in float32 (:3432-3448), then Q4_128 blocks. */
int asdsl_b200_requant_q4_128(const uint8_t* packed, const uint16_t* scales, const uint16_t* zeros, int rows, int cols,
                              uint8_t* blocks, void* stream);

/* Re-lay Q4_128 blocks (repack_q4_128.py:34-92) into the banded device layout: pure byte moves,
 * bit-exact; rows past M in the last band are zero.  quant: ceil(M/4)*(K/128)*256 bytes,
 * scales: ceil(M/4)*(K/128)*8 bytes.  Device-side counterpart of the reference's per-format
 * repackers (asdsl/quantization/repack_q4_128.py, repack_preq2.py:22-46 for the band idea). */
int asdsl_b200_relayout_q4_128(const uint8_t* blocks, uint8_t* quant, uint8_t* scales, int out_features,
                               int in_features, void* stream);

/* Q4_128 GEMV on the banded layout with fused A8 at gs 128: same result as
 * quantize_activation_avx2(..., 128) + gemv_q4_128_preq_avx2 on the original blocks
 * (asdsl/kernels/native/gemv_q4_128.cpp:94-257). */
int asdsl_b200_gemv_q4_128_banded(const uint8_t* quant, const uint8_t* scales, const float* x, float* y,
                                  int out_features, int in_features, void* stream);

/* Bytes of device scratch the fused-argmax GEMVs need (zero-filled once by the caller;
 * the kernels leave it re-armed). */
size_t asdsl_b200_argmax_scratch_bytes(void);

/* lm_head GEMV with fused first-max argmax (fused A8; fmt PREQ2 at gs 32, Q4_128 or Q4_128_BANDED
 * at gs 128; for the banded layout w0 = quant, w1 = scales).
 * Writes logits to y (may be NULL) and the maximum / its global row index (row_base + local row)
 * to out_val[0] / out_idx[0].  Replaces the engine's lm_head GEMV + argmax_f32_avx2
 * (asdsl/kernels/native/unified_engine.cpp:1628-1644 and :207-233). */
int asdsl_b200_gemv_argmax(int fmt, const uint8_t* w0, const uint8_t* w1, const float* x, float* y,
                           float* out_val, int32_t* out_idx, int row_base, void* scratch, size_t scratch_bytes,
                           int out_features, int in_features, void* stream);

/* asdsl_b200_gemv_argmax without caller scratch, for callers that cannot allocate device memory.
 * No counterpart in the reference (its CPU argmax needs no device scratch).
 * The scratch is a file-scope device array of 8448 bytes (one per device), enough for grids of up
 * to 1024 CTAs; a device that would launch more is rejected with ASDSL_B200_ERANGE.  The function
 * allocates nothing.  The FIRST call on each device (with that device current) resolves the array's
 * address with cudaGetSymbolAddress and zeroes it on `stream`; make that first call before any
 * stream capture.  All calls on one device share the array: calls that overlap in time (on two
 * streams, or from two host threads) race and must be serialised by the caller. */
int asdsl_b200_gemv_argmax_static(int fmt, const uint8_t* w0, const uint8_t* w1, const float* x, float* y,
                                  float* out_val, int32_t* out_idx, int row_base, int out_features,
                                  int in_features, void* stream);

/* Row-sharded lm_head across the GPUs of one box (one process per GPU): the argmax of the
 * last CTA is exchanged with the peers inside the kernel (NVLink peer stores of one packed
 * (max, index, step) word per rank into every rank's slot buffer, bounded wait for all words),
 * so every rank ends the kernel holding the global first maximum.  Replaces the engine's
 * lm_head GEMV + argmax_f32_avx2 (asdsl/kernels/native/unified_engine.cpp:1628-1662, :207-233)
 * split over GPUs with an all-gather of (max, index).
 * Setup: each rank calls asdsl_b200_xchg_create (ipc_handle receives
 * asdsl_b200_xchg_handle_bytes() bytes), the handles are all-gathered in rank order by the host
 * (e.g. torch.distributed), and each rank calls asdsl_b200_xchg_open with the world's handles.
 * Every rank must then call asdsl_b200_gemv_argmax_xchg the same number of times; a call whose
 * peers do not arrive within 2 s returns ASDSL_B200_ETIMEOUT through the device status word.
 * Global indices (row_base + local row) must stay below 2^24. */
typedef struct asdsl_b200_xchg asdsl_b200_xchg;
int asdsl_b200_xchg_create(int world, int rank, asdsl_b200_xchg** out, void* ipc_handle);
size_t asdsl_b200_xchg_handle_bytes(void);
int asdsl_b200_xchg_open(asdsl_b200_xchg* xchg, const void* handles);
int asdsl_b200_xchg_destroy(asdsl_b200_xchg* xchg);
/* Optional instrumentation: each later asdsl_b200_gemv_argmax_xchg writes four %globaltimer
 * stamps (ns) of step e to stamps[(e & (n_slots - 1)) * 4 + i]: i = 0 the consumers released
 * (previous kernel complete, CTA 0), 1 the local argmax reduced (last CTA), 2 this rank's word
 * stored to every peer, 3 every peer's word seen.  `stamps` is device memory of n_slots * 4
 * words, n_slots a power of two; null turns the stamps off.  No reference counterpart. */
int asdsl_b200_xchg_set_stamps(asdsl_b200_xchg* xchg, unsigned long long* stamps, int n_slots);
int asdsl_b200_gemv_argmax_xchg(int fmt, const uint8_t* w0, const uint8_t* w1, const float* x, float* y,
                                float* out_val, int32_t* out_idx, int row_base, void* scratch,
                                size_t scratch_bytes, int out_features, int in_features, asdsl_b200_xchg* xchg,
                                void* stream);

/* Row-sharded MLP across the GPUs of one box (one process per GPU): rank r holds gate/up rows
 * [a_r, b_r) and the matching input columns of down_proj, so each rank's down GEMV yields a
 * partial of the hidden vector; asdsl_b200_allreduce_peer sums the partials of all ranks in one
 * kernel: NVLink peer stores of this rank's partial into every rank's buffer as 64-bit words
 * (the float and the step number, so no fence or flag is needed), then a bounded wait on each
 * word and a rank-ordered sum -- every rank gets the same bits -- optionally adding a residual:
 * out = (sum over r of part_r) + add.  Replaces the down projection of the engine's MLP
 * (asdsl/kernels/native/unified_engine.cpp:1586-1597) split over GPUs with an all-reduce.
 * Setup as for asdsl_b200_xchg: create on every rank (ipc_handle receives
 * asdsl_b200_vxchg_handle_bytes() bytes; world <= 16), all-gather the handles in rank order,
 * open.  Every rank must call asdsl_b200_allreduce_peer the same number of times with the same
 * n (<= n_max); `part` and `out` must not overlap; a call whose peers do not arrive within 2 s
 * sets the device status word (ASDSL_B200_ETIMEOUT from asdsl_b200_device_status). */
typedef struct asdsl_b200_vxchg asdsl_b200_vxchg;
int asdsl_b200_vxchg_create(int world, int rank, int n_max, asdsl_b200_vxchg** out, void* ipc_handle);
size_t asdsl_b200_vxchg_handle_bytes(void);
int asdsl_b200_vxchg_open(asdsl_b200_vxchg* vxchg, const void* handles);
int asdsl_b200_vxchg_destroy(asdsl_b200_vxchg* vxchg);
/* Optional instrumentation as asdsl_b200_xchg_set_stamps, per asdsl_b200_allreduce_peer step
 * (CTA 0): 0 kernel start (previous kernel complete), 1 own partial stored to its peer, 2 CTA 0's
 * slice gathered from every rank and summed, 3 the step counter advanced.  The setting lives in
 * device memory, so it also reaches steps replayed from CUDA graphs captured earlier; call it
 * while no step of this exchange runs. */
int asdsl_b200_vxchg_set_stamps(asdsl_b200_vxchg* vxchg, unsigned long long* stamps, int n_slots);
int asdsl_b200_allreduce_peer(asdsl_b200_vxchg* vxchg, const float* part, float* out, const float* add, int n,
                              void* stream);

/* Fused gate_up GEMV + SiLU(gate)*up: rows [0, I) are gate, [I, 2I) are up, h[i] = silu(gate_i)*up_i
 * with the reference's fast_exp.  fmt PREQ2 (w0 = meta, w1 = quant), Q4_128 (w0 = blocks) or
 * Q4_128_BANDED (w0 = quant, w1 = scales).
 * Replaces the gate_up GEMV + swiglu_inplace pair (asdsl/kernels/native/unified_engine.cpp:1539-1570,
 * :836-857). */
int asdsl_b200_gateup_silu(int fmt, const uint8_t* w0, const uint8_t* w1, const float* x, float* h,
                           int intermediate, int in_features, void* stream);

/* Multi-token W4A8 GEMV (speculative verification): Y[t][M] = W . A8(X[t][K]) for t < n_tokens,
 * each row exactly the single-token result.  Replaces the per-token loop of the verify path
 * (forward_verify_serial, asdsl/kernels/native/unified_engine.cpp:1766-1772, over
 * gemv_q4_32_preq_fused_avx2 / gemv_q4km_q8_avx2) and the batched gemm_q4_32_q8_avx2
 * (asdsl/kernels/native/gemm_batch.cpp:146-260).  fmt PREQ (w0 = blocks), PREQ2 (w0 = meta,
 * w1 = quant), Q4_128_BANDED (w0 = quant, w1 = scales; A8 at gs 128) or Q4K (w0 = blocks, the
 * Q4_K kernel's own A8).  Up to 16 tokens share one weight stream (fewer when 16 A8 rows of
 * in_features do not fit beside the pipeline); more tokens take further passes. */
int asdsl_b200_gemv_multi(int fmt, const uint8_t* w0, const uint8_t* w1, const float* X, float* Y,
                          int out_features, int in_features, int n_tokens, void* stream);

/* One decoder layer's projection set (the config-1 workload) behind a synchronous host-buffer
 * call: qkv = W_qkv x and o = W_o qkv[:q_dim] (preq2 gs 32), h = SiLU(W_gate o) * (W_up o) and
 * y = W_down h (banded Q4_128) -- the reference runs these as the projections of
 * UnifiedEngine::forward_token (asdsl/kernels/native/unified_engine.cpp:1411-1413, :1487-1489,
 * :1532-1538, :1592-1598), each a call of its native GEMV from the host.
 * layer_create borrows the device weights and the device buffers x_dev[hidden], h_dev[inter] and
 * out_dev[qkv_rows + 2 * hidden] (qkv | o | y), which must outlive the handle; it makes its own
 * stream and pinned staging, runs one step and captures the step as one CUDA graph: a kernel
 * reading x from the pinned staging (mapped host memory), the four GEMVs, a kernel writing
 * out_dev to the pinned staging.  layer_forward copies x_host[hidden] in, replays the graph,
 * waits, and copies the results to out_host[qkv_rows + 2 * hidden]; one call at a time per
 * handle. */
typedef struct asdsl_b200_layer asdsl_b200_layer;
int asdsl_b200_layer_create(const uint8_t* qkv_meta, const uint8_t* qkv_quant, const uint8_t* o_meta,
                            const uint8_t* o_quant, const uint8_t* gu_quant, const uint8_t* gu_scales,
                            const uint8_t* dn_quant, const uint8_t* dn_scales, float* x_dev, float* h_dev,
                            float* out_dev, int hidden, int qkv_rows, int q_dim, int inter, asdsl_b200_layer** out);
int asdsl_b200_layer_forward(asdsl_b200_layer* layer, const float* x_host, float* out_host);
int asdsl_b200_layer_destroy(asdsl_b200_layer* layer);

/* Small host <-> device transfers as kernels (no counterpart in the reference, whose kernels take
 * host arrays directly): host_pinned must be pinned host memory (cudaMallocHost, cudaHostAlloc,
 * torch's pin_memory), which the kernel reads or writes through its mapped address; both buffers
 * 16-byte aligned (others are rejected with ASDSL_B200_EINVAL).  For a few
 * KB this costs ~1 us where a copy-engine transfer costs ~10 us; device_to_host launches with
 * programmatic dependent launch and waits for the previous kernel on the stream.  Stream-ordered;
 * the host sees device_to_host's data after synchronizing the stream. */
int asdsl_b200_host_to_device(const float* host_pinned, float* dev, long long n, void* stream);
int asdsl_b200_device_to_host(const float* dev, float* host_pinned, long long n, void* stream);

/* Reference-exact GEMVs (see ASDSL_B200_NUMERICS_REFERENCE_EXACT): gemv_preq2_fused_avx2
 * (gemv_preq2_avx2.cpp:301-319) with every row summed as the compiled process_one_row does
 * (:216-253), bit-identical to the reference kernel.  norm_w non-null folds the engine's
 * preceding rmsnorm_f32(x) * norm_w in first (unified_engine.cpp:499-524, RSQRTSS + Newton as
 * compiled; in_features % 8 == 0).  gateup_silu_exact: the gate_up GEMV (rows [0, 2I)) followed
 * by swiglu_inplace (:836-857, RCPPS + Newton as compiled) -> h[I]. */
int asdsl_b200_gemv_preq2_fused_exact(const uint8_t* meta, const uint8_t* quant, const float* x, const float* norm_w,
                                      float eps, float* y, int M, int K, void* stream);
int asdsl_b200_gateup_silu_exact(const uint8_t* meta, const uint8_t* quant, const float* x, const float* norm_w,
                                 float eps, float* h, int I, int K, void* stream);
/* Builds (once per process) the host tables of the reference-exact mode and uploads them to
 * the current device; *n_exp_exceptions = number of inputs where the C library's expf is not
 * the correctly rounded exp.  asdsl_b200_exact_host_tables copies the host tables out (tests):
 * rcp[2048], rsqrt[2048], exp_exc[2 * n] (input bits, expf bits) when exp_cap >= n. */
int asdsl_b200_exact_numerics_init(int* n_exp_exceptions);
int asdsl_b200_exact_host_tables(uint32_t* rcp, uint32_t* rsqrt, uint32_t* exp_exc, int exp_cap, int* n_exp);
/* The attention's expf of the reference-exact mode over a device array (x <= 0; tests): the
 * C library's expf (unified_engine.cpp:989, :1000) bit for bit. */
int asdsl_b200_exact_expf(const float* x, float* y, long long n, void* stream);

/* ======================================================================================
 * Device-resident decode engine: UnifiedEngine (asdsl/kernels/native/unified_engine.h:14-109,
 * :134-282; unified_engine.cpp) for the C0 decode path.  The engine owns its device memory
 * (weights re-laid out on upload, int8 KV cache, activations) and one CUDA stream; a decode
 * step is one CUDA-graph replay.  Every setter accepts host or device pointers (copied).
 * ==================================================================================== */

/* EngineConfig (unified_engine.h:14-109, pybind fields unified_engine.cpp:2204-2222).
 * Supported here: head_dim 128, weight_format 0 with group_size 32, lm_head_group_size 32 or 128
 * (0 = group_size), hidden / intermediate / q dims multiples of 128. */
typedef struct asdsl_b200_engine_config {
    int num_layers;
    int hidden_size;
    int num_heads;
    int num_kv_heads;
    int head_dim;
    int intermediate_size;
    int vocab_size;
    float rms_norm_eps;
    int group_size;
    int lm_head_group_size;
    int max_seq_len;
    int rotary_dim;
    int weight_format;
} asdsl_b200_engine_config;

typedef struct asdsl_b200_engine asdsl_b200_engine;

/* UnifiedEngine constructor, split into create + setters + finalize
 * (pybind constructor unified_engine.cpp:2662-2682, weight binding :2240-2442). */
int asdsl_b200_engine_create(const asdsl_b200_engine_config* cfg, asdsl_b200_engine** out);
int asdsl_b200_engine_destroy(asdsl_b200_engine* e);
/* token_embd [vocab][hidden] fp16 (embd_is_f16 = 1) or fp32; output_norm [hidden];
 * cos/sin tables [max_seq_len][rotary_dim/2] fp32. */
int asdsl_b200_engine_set_globals(asdsl_b200_engine* e, const void* token_embd, int embd_is_f16,
                                  const float* output_norm, const float* cos_table, const float* sin_table);
/* lm_head source [vocab][hidden] fp16 or fp32, quantized on the device at finalize with the
 * reference constructor's rules (unified_engine.cpp:320-400 g32 -> preq2, :411-461 g128). */
int asdsl_b200_engine_set_output_proj(asdsl_b200_engine* e, const void* output_proj, int is_f16);
/* Cached lm_head preq2 blobs (unified_engine.cpp:295-318): used when lm_head_group_size is 32
 * and both sizes match, otherwise ignored as the reference does. */
int asdsl_b200_engine_set_lm_head_preq2(asdsl_b200_engine* e, const uint8_t* meta, size_t meta_bytes,
                                        const uint8_t* quant, size_t quant_bytes);
/* layers_dict[i]["rms_att"], ["rms_ffn"]  (unified_engine.cpp:2306-2320). */
int asdsl_b200_engine_set_layer_norms(asdsl_b200_engine* e, int layer, const float* rms_att, const float* rms_ffn);
/* layers_dict[i] projection weights: which 0 qkv, 1 o, 2 gate_up (gate rows then up rows), 3 down.
 * fmt PREQ2 (w0 = *_meta, w1 = *_quant; unified_engine.cpp:2368-2386) or Q4_128 (w0 = *_g128 blocks,
 * re-laid out to the banded device layout; :2330-2349). */
int asdsl_b200_engine_set_projection(asdsl_b200_engine* e, int layer, int which, int fmt, const uint8_t* w0,
                                     size_t w0_bytes, const uint8_t* w1, size_t w1_bytes);
/* Builds the lm_head, runs one eager step and captures the decode / prefill graphs. */
int asdsl_b200_engine_finalize(asdsl_b200_engine* e);
/* forward_token (unified_engine.cpp:1339-1688; pybind :2485-2510): logits (host or device, vocab floats)
 * and / or argmax may be NULL; both NULL = forward_token_prefill (no lm_head).
 * token / pos out of range -> ASDSL_B200_ERANGE. */
int asdsl_b200_engine_forward_token(asdsl_b200_engine* e, int token, int pos, float* logits, int32_t* argmax);
/* forward_verify_serial (unified_engine.cpp:1767-1772; pybind forward_verify_serial_all_logits
 * :2602-2611, and forward_batch_all_logits :2591-2600, which takes the serial path under preq2,
 * :1774-1789): forward_token(tokens[i], start_pos + i) for i < n; out_logits (host or device) receives
 * n x vocab floats, row i = the logits of step i.  n <= 0 is a no-op; a token or position out of range
 * -> ASDSL_B200_ERANGE before any step runs. */
int asdsl_b200_engine_forward_verify(asdsl_b200_engine* e, const int32_t* tokens, int n, int start_pos,
                                     float* out_logits);
/* forward_batch (unified_engine.cpp:1117; pybind forward_batch :2526-2534 with all_logits = 0, and
 * forward_verify_batch_raw_all_logits :2613-2625 with all_logits = 1): tokens[i] at position
 * start_pos + i for i < n, passes of up to 16 tokens, each sharing one weight read per projection
 * (multi-token GEMVs).  out_logits (host or device; may be NULL) receives the last token's vocab
 * logits, or n x vocab rows when all_logits != 0.  Logits and KV cache are bit-identical to n
 * forward_token calls of the per-op decode chain (the reference's batched GEMM path is not: its
 * binding documents that it may diverge).  Ranges as forward_verify. */
int asdsl_b200_engine_forward_batch(asdsl_b200_engine* e, const int32_t* tokens, int n, int start_pos,
                                    float* out_logits, int all_logits);
/* generate / generate_with_stops (unified_engine.cpp:1717-1764): out = prompt + generated tokens
 * (the stop token included), *n_out its length; out_cap >= n_prompt + max_tokens + 1.  The prompt
 * tokens but the last are forwarded in batched passes (the forward_batch arithmetic, bit-identical
 * to per-token forwards), the rest one decode-graph replay per token. */
int asdsl_b200_engine_generate(asdsl_b200_engine* e, const int32_t* prompt, int n_prompt, int max_tokens,
                               const int32_t* stops, int n_stops, int32_t* out, int out_cap, int* n_out);
/* reset_session / get_kv_seq_len / truncate_kv / snapshot_kv / restore_kv (unified_engine.cpp:1285-1337). */
int asdsl_b200_engine_reset_session(asdsl_b200_engine* e);
int asdsl_b200_engine_get_kv_seq_len(asdsl_b200_engine* e, int* out);
int asdsl_b200_engine_truncate_kv(asdsl_b200_engine* e, int new_len);
int asdsl_b200_engine_snapshot_kv(asdsl_b200_engine* e);
int asdsl_b200_engine_restore_kv(asdsl_b200_engine* e);
/* export_lm_head_preq2 (unified_engine.cpp:2470-2483): *fmt = PREQ2 (w0 meta, w1 quant) or
 * Q4_128_BANDED (w0 quant, w1 scales); NULL buffers = format query only. */
int asdsl_b200_engine_export_lm_head(asdsl_b200_engine* e, int* fmt, uint8_t* w0, size_t w0_bytes, uint8_t* w1,
                                     size_t w1_bytes);
/* Benchmark / graph-level control (no reference counterpart): the engine's stream, stream-ordered
 * setting of (pos, seq[pos] = token; token < 0 leaves seq alone), and n replays of the decode
 * (decode = 1) or prefill graph without synchronising. */
int asdsl_b200_engine_stream(asdsl_b200_engine* e, void** stream);
/* Decode-step implementation, chosen before finalize: persistent = 0 (default) runs the per-op
 * kernel chain (163 kernels per token in one CUDA graph, chained by programmatic dependent
 * launch); 1 runs each step as one cooperative kernel over a program of ops with grid barriers
 * between them.  The environment variable ASDSL_B200_DECODE_KERNEL=persistent selects 1 at
 * create. */
/* Sharded decode across the GPUs of one box (one process and one engine per GPU): call after
 * asdsl_b200_engine_create and before the lm_head and projections are set.  The engine then
 * holds this rank's slice of every layer's MLP -- config.intermediate_size gate rows and the
 * matching up rows (gate_up = local gate rows then local up rows) and down_proj's matching input
 * columns -- and rows [lm_row_base, lm_row_base + lm_rows) of the lm_head (set_output_proj /
 * set_lm_head_preq2 take those rows only).  Each layer's down partial is summed over the ranks
 * by asdsl_b200_allreduce_peer (with the residual add); the lm_head argmax is exchanged inside
 * its kernel (asdsl_b200_gemv_argmax_xchg), so every rank produces the same tokens.  qkv, o and
 * attention are replicated.  Fast numerics and the per-op chain only; forward_token returns the
 * argmax (no logits), forward_batch / forward_verify / export_lm_head are not available.
 * finalize, forward_token and generate run exchange steps: every rank makes the same calls.
 * Replaces the reference engine's MLP and lm_head (asdsl/kernels/native/unified_engine.cpp:
 * 1532-1598, :1628-1662) split over GPUs. */
int asdsl_b200_engine_set_shard(asdsl_b200_engine* engine, asdsl_b200_vxchg* vxchg, asdsl_b200_xchg* xchg,
                                int lm_rows, int lm_row_base);

/* Draft steps (QCSD / SWIFT self-speculation, unified_engine.cpp:1790-1802, :1309-1322):
 * set_skip_mask(mask, n) -- layers l < n with mask[l] != 0 are left out of draft steps (the
 * reference's set_skip_mask; reset_session clears it, as there); set_projection_q2 -- the layer's
 * 2-bit draft-bank projection (which: 0 qkv, 1 o, 2 gate_up, 3 down; packed codes [rows][cols/4],
 * fp32 scales / biases [rows][cols/32]; the layers_dict keys q2_{qkv,o,gate_up,down}_{proj,scales,
 * biases}, unified_engine.cpp:2387-2440); forward_token_draft -- one decode step at (token, pos) with
 * the masked layers left out (forward_token_draft) and, with use_q2, the 2-bit projections in place
 * of the 4-bit ones where set (forward_token_draft_q2), logits and/or argmax as forward_token.
 * Fast numerics on one GPU (not with the reference-exact mode, the persistent kernel or a shard). */
int asdsl_b200_engine_set_skip_mask(asdsl_b200_engine* engine, const uint8_t* mask, int n);
int asdsl_b200_engine_clear_skip_mask(asdsl_b200_engine* engine);
int asdsl_b200_engine_set_projection_q2(asdsl_b200_engine* engine, int layer, int which, const uint8_t* w_packed,
                                        size_t w_bytes, const float* scales, const float* biases, size_t n_groups);
int asdsl_b200_engine_forward_token_draft(asdsl_b200_engine* engine, int token, int pos, float* logits,
                                          int32_t* argmax, int use_q2);

/* Numerics of the decode step, set before finalize (no reference switch: the reference has one
 * numerics, its compiled code's).  ASDSL_B200_NUMERICS_FAST: the streaming kernels' own fp32
 * summation order (every GEMV within 1e-3 of the reference; the default).
 * ASDSL_B200_NUMERICS_REFERENCE_EXACT: every op in the operation order of the reference's
 * -ffast-math build -- forward_token (unified_engine.cpp:1339-1688) with process_one_row's
 * 8-lane accumulators (gemv_preq2_avx2.cpp:216-253), rmsnorm_f32's RSQRTSS + Newton step
 * (:499-524), swiglu_inplace's RCPPS + Newton step (:836-857), set_kv_cache's 127/absmax
 * (:859-920) and attention's C-library expf (:922-1027) -- so logits and greedy tokens are
 * bit-identical to the reference's on this host.  Needs an x86 host (the approximate-reciprocal
 * and expf tables are captured from its CPU and C library on first use: about a second), preq2
 * gs 32 weights, head_dim 128 and max_seq_len <= 4096; forward_batch runs serial steps. */
#define ASDSL_B200_NUMERICS_FAST 0
#define ASDSL_B200_NUMERICS_REFERENCE_EXACT 1
int asdsl_b200_engine_set_numerics(asdsl_b200_engine* e, int mode);
int asdsl_b200_engine_set_persistent(asdsl_b200_engine* e, int persistent);
/* Per-op profile of one step of the persistent decode kernel at the current position (the
 * device-side counterpart of the reference's ASDSL_ENGINE_PROFILE per-op breakdown,
 * unified_engine.cpp:58-95): host_trace[3*i + {0,1,2}] = earliest start of op i over all CTAs,
 * latest end of its work, latest exit from the grid barrier after it (globaltimer ns).  The
 * step runs eagerly and advances the position like a replay. */
int asdsl_b200_engine_profile_step(asdsl_b200_engine* e, int decode, unsigned long long* host_trace, int max_ops,
                                   int* n_ops);
int asdsl_b200_engine_set_position(asdsl_b200_engine* e, int pos, int token);
int asdsl_b200_engine_replay(asdsl_b200_engine* e, int decode, int n);
/* Copy of an engine buffer to host memory after the engine stream drains (tests only; no reference
 * counterpart): which 0 residual stream, 1 qkv, 2 attention output, 3 SiLU(gate)*up, 4 logits,
 * 5 K codes, 6 V codes, 7 K scales, 8 V scales (the last layer's values for 1-4). */
int asdsl_b200_engine_read_buffer(asdsl_b200_engine* e, int which, void* host, size_t bytes);

#ifdef __cplusplus
}
#endif
#endif /* ASDSL_B200_H */
