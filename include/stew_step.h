/*
 * stew_step.h -- C ABI of the layer kernels around the NF4 projections in the packed-token
 * QLoRA step (same library and conventions as stew_nf4.h: device pointers, sizes in elements,
 * `void* stream` = cudaStream_t, int status, no allocation, no host synchronisation).
 *
 * They stand in for the reference's Triton kernels of the same Qwen2 layer:
 *   nf4b_rmsnorm_fwd (delta == NULL) <- solution/rmsnorm.py:19-34  _rms_fwd
 *   nf4b_rmsnorm_fwd (delta given)   <- solution/rmsnorm.py:152-168 _add_rms_fwd
 *   nf4b_rmsnorm_bwd (dsum NULL/set) <- solution/rmsnorm.py:36-50 _rms_bwd, :171-190 _add_rms_bwd
 *   nf4b_rope_qk                     <- solution/rope.py:24-52 rope_kernel (forward, and INVERSE
 *                                       for the backward) applied to q and k in one launch
 *   nf4b_swiglu_fwd / _bwd           <- solution/swiglu.py:15-40
 *   nf4b_ce_fwd / _bwd               <- solution/head_loss.py (loss, then softmax - onehot)
 * Activations are fp16, row-major.
 */
#ifndef STEW_STEP_H
#define STEW_STEP_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* y[r] = fp16(w * fp16(s[r] * rstd[r])), rstd[r] = 1/sqrt(mean(s[r]^2) + eps), where
 * s = x (delta == NULL) or s = fp16(x + delta), then also written to `sum` (the residual
 * stream).  x, delta, sum, y: fp16 [rows, hidden]; w: fp32 [hidden]; rstd: fp32 [rows].
 * hidden must be a multiple of 256 and at most 4096.  */
int nf4b_rmsnorm_fwd(const void* x, const void* delta, const float* w, float eps, void* sum,
                     void* y, float* rstd, int64_t rows, int64_t hidden, void* stream);

/* dx = rstd * (w*dy - xn * mean(w*dy*xn)) (+ dsum), xn = x * rstd: the input gradient of
 * nf4b_rmsnorm_fwd (x = the normalised input s); with the fused add, dsum is the gradient
 * arriving at `sum`, and dx is the gradient of both x and delta.  */
int nf4b_rmsnorm_bwd(const void* dy, const void* x, const float* w, const float* rstd,
                     const void* dsum, void* dx, int64_t rows, int64_t hidden, void* stream);

/* Rotary embedding (rotate-half convention, fp32 math) on q [tokens, q_heads, head_dim] and
 * k [tokens, k_heads, head_dim] with cos/sin fp32 [tokens, head_dim]:
 *   out[i] = x[i] cos[i] - x[i+d] sin[i],   out[i+d] = x[i+d] cos[i+d] + x[i] sin[i+d],
 * d = head_dim/2; inverse != 0 applies the transposed rotation (the backward).
 * head_dim must be a multiple of 16; either tensor may be skipped with 0 heads.  */
int nf4b_rope_qk(const void* q, const void* k, const float* cos_t, const float* sin_t, void* q_out,
                 void* k_out, int64_t tokens, int32_t q_heads, int32_t k_heads, int32_t head_dim,
                 int32_t inverse, void* stream);

/* m = fp16(gate * sigmoid(gate) * up), fp32 inside (the reference's SwiGLU kernel,
 * solution/swiglu.py:16-23), n elements (a multiple of 8).  */
int nf4b_swiglu_fwd(const void* gate, const void* up, void* out, int64_t n, void* stream);

/* dup = fp16(dout * gate * sig), dgate = fp16(dout * up * sig * (1 + gate * (1 - sig))),
 * sig = sigmoid(gate), fp32 inside (solution/swiglu.py:26-37).  */
int nf4b_swiglu_bwd(const void* dout, const void* gate, const void* up, void* dgate, void* dup,
                    int64_t n, void* stream);

/* Next-token cross-entropy of the LM head over fp16 logits [rows, vocab] (vocab a multiple of
 * 8, rows 16-byte aligned) with int64 labels [rows] -- the reference's fused head loss
 * (solution/head_loss.py: per-row loss, then the gradient softmax - onehot in place):
 *   nf4b_ce_fwd: loss[r] = logsumexp(logits[r]) - logits[r, labels[r]] (fp32; 0 where the
 *                label is outside [0, vocab), e.g. -100), lse[r] = logsumexp(logits[r]);
 *   nf4b_ce_bwd: logits[r, j] <- fp16(g * (exp(logits[r, j] - lse[r]) - [j == labels[r]])) in
 *                place, g = *gscale (device fp32), zero rows for ignored labels.  */
int nf4b_ce_fwd(const void* logits, const int64_t* labels, float* loss, float* lse, int64_t rows,
                int64_t vocab, void* stream);
int nf4b_ce_bwd(void* logits, const int64_t* labels, const float* lse, const float* gscale,
                int64_t rows, int64_t vocab, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* STEW_STEP_H */
