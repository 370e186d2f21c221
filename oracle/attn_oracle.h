/*
 * attn_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C CPU restatement of the reference engine's per-layer attention step
 * (rain1201/picolm_qwen).  It is the checker that the CUDA path in
 * picolm_qwen_b200/csrc is compared against; nothing in the product links or
 * calls it.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * leg may load the shared object built from this file.
 *
 * Parity pins: tests/test_oracle_golden.py checks every function here against
 * fixtures produced by the reference's own code (oracle/ref_harness.cpp drives
 * the unmodified Model::forward from cpp/model.hpp), bit for bit.
 */
#ifndef PICO_ATTN_ORACLE_H
#define PICO_ATTN_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* fp32 -> fp16 bits with the reference's rounding (cpp/quant.hpp:102-135). */
uint16_t ora_f32_to_f16(float f);
/* fp16 bits -> fp32, exact (cpp/quant.hpp:73-100). */
float ora_f16_to_f32(uint16_t h);
void ora_f32_to_f16_n(const float* in, uint16_t* out, size_t n);
void ora_f16_to_f32_n(const uint16_t* in, float* out, size_t n);

/* In-place per-head RMSNorm in the reference's summation order
 * (cpp/tensor.hpp:146-176, eps 1e-6 hard-coded there). */
void ora_rmsnorm_inplace(float* x, const float* w, int n, float eps);

/* RoPE, NeoX half split (cpp/tensor.hpp:201-283, picolm/tensor.c:221-244). */
void ora_rope_neox(float* q, float* k, int hd, int hq, int hkv,
                   const float* cos_row, const float* sin_row);
/* RoPE, interleaved pairs (picolm/tensor.c:247-293 scalar definition). */
void ora_rope_interleaved(float* q, float* k, int hd, int hq, int hkv,
                          const float* cos_row, const float* sin_row);

/* RoPE table [max_seq][hd/2] (cpp/model.hpp:1008-1017). */
void ora_rope_table(float* cos_t, float* sin_t, int max_seq, int hd, float base);

/*
 * One decode step for one sequence in one layer (cpp/model.hpp:326-418).
 *   q   [hq*hd]  fp32, rotated in place (norm + RoPE applied)
 *   k   [hkv*hd] fp32, rotated in place
 *   v   [hkv*hd] fp32
 *   qn_w, kn_w   [hd] QK-RMSNorm weights or NULL (no norm)
 *   kc, vc       this layer's cache slabs [max_seq][hkv*hd] fp16 bits; row pos is written
 *   out [hq*hd]  attention output
 *   variant 0 = C++ engine update order (cpp/model.hpp:375-418),
 *           1 = C engine update order  (picolm/model.c:781-825)
 * Returns 0, or -1 on invalid arguments.
 */
int ora_decode_step(int hq, int hkv, int hd, int rope_mode, float eps,
                    float* q, float* k, const float* v,
                    const float* qn_w, const float* kn_w,
                    const float* cos_row, const float* sin_row,
                    uint16_t* kc, uint16_t* vc, int pos, float* out, int variant);

/* ora_decode_step variant 0 with the q heads spread over n_threads host
 * threads (same per-head arithmetic); for long single sequences. */
int ora_decode_step_mt(int hq, int hkv, int hd, int rope_mode, float eps,
                       float* q, float* k, const float* v,
                       const float* qn_w, const float* kn_w,
                       const float* cos_row, const float* sin_row,
                       uint16_t* kc, uint16_t* vc, int pos, float* out, int n_threads);

/*
 * Attention only over rows [row_begin, row_end) of an already-filled cache,
 * returning the un-normalised online-softmax state per q head:
 *   m[hq] (running max of score), l[hq] (sum of exp), acc[hq*hd].
 * Same update order as ora_decode_step variant 0; used to check split-KV
 * partials and the log-sum-exp merge.
 */
void ora_attend_rows(int hq, int hkv, int hd, const float* q_rot,
                     const uint16_t* kc, const uint16_t* vc,
                     int row_begin, int row_end,
                     float* m, float* l, float* acc);

/*
 * Prefill of n_tok tokens starting at start_pos for one layer
 * (cpp/model.hpp:493-593: every token runs the decode step at pos = start+i).
 *   q [n_tok][hq*hd], k/v [n_tok][hkv*hd] fp32 (pre-norm, pre-RoPE), not modified
 *   out [n_tok][hq*hd]
 */
int ora_prefill(int hq, int hkv, int hd, int rope_mode, float eps,
                const float* q, const float* k, const float* v,
                const float* qn_w, const float* kn_w,
                const float* cos_t, const float* sin_t,
                uint16_t* kc, uint16_t* vc, int start_pos, int n_tok,
                float* out, int n_threads);

/*
 * Batched decode over B independent sequences, each with its own cache slab,
 * spread over n_threads host threads (one sequence per task).  Arithmetic per
 * head is the single-sequence step above; used for the all-cores CPU baseline.
 *   q [B][hq*hd], k/v [B][hkv*hd] (copied, not modified), kc/vc[b] slab pointers,
 *   pos [B], out [B][hq*hd].
 */
int ora_decode_batch(int B, int hq, int hkv, int hd, int rope_mode, float eps,
                     const float* q, const float* k, const float* v,
                     const float* qn_w, const float* kn_w,
                     const float* cos_t, const float* sin_t,
                     uint16_t* const* kc, uint16_t* const* vc,
                     const int* pos, float* out, int n_threads);

/*
 * Projections around the attention step (TensorOps::matmul_bias,
 * cpp/tensor.hpp:110-143) for the weight formats the C++ engine multiplies
 * with.  type: GGUF tensor type (1 F32, 2 F16, 3 Q4_0, 9 Q8_0, 13 Q4_K,
 * 15 Q6_K; cpp/quant.hpp:16-31).
 */
/* Weights per block and bytes per block (cpp/quant.hpp:137-166); 0 if unsupported. */
int ora_weight_block(int type, int* elems, int* bytes);
/* One row of n weights to fp32 (dequantize_row, cpp/quant.hpp:175-295). */
void ora_dequant_row(const void* src, float* dst, int n, int type);
/* W[row] . x in the reference's order (vec_dot, cpp/quant.hpp:304-358: the
 * SSE2 two-accumulator order for F32 and the dequantised formats, per-block
 * scalar sums for Q8_0). */
float ora_vec_dot(const void* row, const float* x, int n, int type);
/* out[v*n_out + d] = W[d].x[v] (+ bias[d]), or added to out (accumulate):
 * matmul_bias then vec_add (cpp/model.hpp:420-427). */
void ora_matvec(const void* w, int type, const float* bias, int n_in, int n_out, int n_vec,
                const float* x, float* out, int accumulate);

#ifdef __cplusplus
}
#endif
#endif
