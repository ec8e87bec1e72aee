/*
 * qmm_oracle.h -- CPU restatement of the reference's GGUF quantized-matmul
 * path (openIE-dev/rce, crates rce-op-qmm, rce-ingest-gguf, rce-op-moe,
 * rce-vm-backend-cpu/src/ml).
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA path
 * is compared against, and the CPU baseline that bench.py times beside it.
 * Nothing in the product (rce_b200/, the C-ABI library) links or calls it.
 *
 * Every function restates one reference function in the same loop order and
 * the same binary32 operation sequence; the file:line it follows is given at
 * each definition in qmm_oracle.c.  Built with -ffp-contract=off and without
 * fast-math, so no FMA contraction and no reassociation happen: on x86-64 the
 * results are bit-identical to the reference's scalar x86 path.
 */
#ifndef RCE_QMM_ORACLE_H
#define RCE_QMM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF dtype tags (rce-ingest-gguf/src/parser.rs:308-338). */
#define ORACLE_GGUF_F32 0
#define ORACLE_GGUF_F16 1
#define ORACLE_GGUF_Q4_0 2
#define ORACLE_GGUF_Q8_0 8
#define ORACLE_GGUF_Q4_K 12
#define ORACLE_GGUF_Q5_K 13
#define ORACLE_GGUF_Q6_K 14

float oracle_f16_to_f32(uint16_t h);
float oracle_round_to_f16(float x);
uint16_t oracle_f32_to_f16_bits(float x);
void oracle_q4k_get_scale_min(const uint8_t *scales, int j, uint8_t *sc, uint8_t *m);
size_t oracle_tensor_byte_size(int dtype, size_t numel);

/* dequantize_to_f32 for Q4_0 / Q8_0 / Q4_K / Q5_K / Q6_K.  Returns 0, or -1 for an
 * unsupported dtype (the reference returns None). out holds ceil(n/blk)*blk. */
int oracle_dequant(const uint8_t *bytes, size_t nbytes, int dtype, size_t n, float *out);

/* mm_1d: out[j] = a . W[j,:] for rows [row0,row1), nthreads threads over rows
 * (rayon's split).  Returns -1 for an unsupported dtype (reference panics). */
int oracle_mm_1d_rows(const float *a, const uint8_t *w, int dtype, size_t n_rows,
                      size_t n_cols, size_t row0, size_t row1, float *out, int nthreads);
int oracle_mm_1d(const float *a, const uint8_t *w, int dtype, size_t n_rows,
                 size_t n_cols, float *out, int nthreads);
/* mm_batched: T x mm_1d (rce-op-qmm/src/lib.rs:1015-1021). */
int oracle_mm_batched(const float *a, size_t t_rows, const uint8_t *w, int dtype,
                      size_t n_rows, size_t n_cols, float *out, int nthreads);

/* moe_router on given logits (rce-op-moe/src/lib.rs:49-72). */
void oracle_moe_softmax_topk(const float *logits, int n_experts, int top_k, int normalize,
                             int32_t *idx, float *weights);
/* moe_router with the gate projection (rce-op-moe/src/lib.rs:35-73). */
int oracle_moe_router(const float *x, const uint8_t *gate_w, int gate_dtype, int n_experts,
                      size_t d_model, int top_k, int normalize, int32_t *idx, float *weights);
/* moe_combine (rce-op-moe/src/lib.rs:98-110); outs is [k][d_model]. */
void oracle_moe_combine(const float *weights, int k, const float *outs, size_t d_model, float *out);
float oracle_silu(float x);
/* Expert-grouped SwiGLU FFN over T tokens with given router logits [T][E]:
 * per token route, per routed expert g = W_gate x, u = W_up x, h = silu(g) u,
 * y = W_down h (rce-qwen36-moe/src/lib.rs:666-705), combine in route order.
 * Expert e's weights are gate + e*gate_stride etc.  out is [T][d_model]. */
int oracle_moe_ffn(const float *x, size_t t_rows, size_t d_model, size_t d_ff,
                   const float *router_logits, int n_experts, int top_k,
                   const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                   size_t gate_stride, size_t up_stride, size_t down_stride, int dtype,
                   float *out, int nthreads);

/* GGUF reference quantizer for one block of 32 (rce-vm-backend-cpu/src/ml/nn.rs:541-563). */
void oracle_quantize_block(const float *x, int q4, int32_t *q, float *d);

/* Spec kernels on unpacked values (rce-vm-backend-cpu/src/ml/nn.rs:477-517,
 * ml/kquant.rs:81-150): an independent restatement of the normative order. */
void oracle_spec_matmul_q(const float *x, size_t m, const int32_t *q, const float *d,
                          size_t n, size_t k, int q4, float *out);
void oracle_spec_matmul_q4k(const float *x, size_t m, const int32_t *q, const float *s,
                            const float *o, size_t n, size_t k, float *out);

/* Reference-test activation generators, evaluated in binary32 with libm's
 * sinf/cosf as Rust's f32::sin/cos do on this platform:
 *   kind 0: sin(i*c1 + c0)    kind 1: cos(i*c1 + c0)   (i as f32 * c1 + c0). */
void oracle_test_activations(int kind, float c1, float c0, size_t n, float *out);

#ifdef __cplusplus
}
#endif
#endif
