/*
 * stew_nf4.h -- C ABI of the B200 (sm_100a) NF4 hot path.
 *
 * Every entry point takes raw device pointers, sizes and a CUDA stream handle
 * (cudaStream_t passed as void*; NULL = legacy default stream), enqueues its
 * kernels on that stream and returns a status code (NF4B_OK == 0).  None of
 * them synchronises the stream or allocates device memory; the caller owns
 * every buffer.  Inputs outside the supported envelope return
 * NF4B_ERR_UNSUPPORTED without launching anything, so a caller can route them
 * to another implementation (the reference does the same: nf4.py:61-70 guard,
 * nf4.py:112 fallback).
 *
 * The functions mirror the reference's Python interface (evilandangry/stew,
 * solution/nf4.py) as follows:
 *   nf4b_dequant          <- dequantize_nf4(A, st)             nf4.py:73-92
 *                            (the launch of _nf4_unpack,       nf4.py:30-50)
 *   nf4b_dequant_batched  <- 196 x dequantize_nf4 per step     tools/bench_nf4.py:47
 *   nf4b_linear_fwd       <- patched MatMul4Bit.forward        nf4.py:142-159
 *                            (unpack + F.linear, nf4.py:148-152) fused, plus the
 *                            peft lora.Linear q/v term y += (x A^T) B^T * s
 *   nf4b_linear_bwd_dx    <- bitsandbytes MatMul4Bit.backward grad_A = dY . W
 *                            on the re-dequantised weight      nf4.py:102-112, :131-133
 *                            plus the LoRA input-gradient term
 *   nf4b_lora_grads       <- peft LoRA weight grads (autograd through lora_A/lora_B)
 */
#ifndef STEW_NF4_H
#define STEW_NF4_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum nf4b_status {
  NF4B_OK = 0,
  NF4B_ERR_INVALID_ARG = 1,  /* NULL pointer, negative or inconsistent size */
  NF4B_ERR_UNSUPPORTED = 2,  /* outside the envelope (blocksize, dtype, shape); nothing launched */
  NF4B_ERR_ALIGNMENT = 3,    /* a pointer or row stride the kernel needs aligned is not */
  NF4B_ERR_CUDA = 4,         /* a CUDA runtime call or a launch failed */
  NF4B_ERR_DEVICE = 5        /* current device is not an sm_100 part */
};

enum nf4b_dtype { NF4B_F16 = 0, NF4B_F32 = 1 };

/* The fields of a bitsandbytes QuantState the unpack reads (nf4.py:61-70, :80-91).
 * Nested (double-quantized) state:
 *   scale[r] = code2[absmax8[r]] * absmax2[r / blocksize2] + offset[0]
 * Plain state:
 *   scale[r] = absmax32[r]
 * value = code[nibble] * scale[r], fp32, rounded once to the output dtype.  */
typedef struct nf4b_qstate {
  const uint8_t* absmax8;   /* nested: 8-bit absmax codes, one per block      */
  const float* absmax32;    /* plain: fp32 absmax, one per block             */
  const float* code2;       /* nested: 256-entry fp32 second-level code      */
  const float* absmax2;     /* nested: fp32, one per blocksize2 blocks       */
  const float* offset;      /* nested: one fp32 on the device (QuantState.offset) */
  const float* code;        /* 16-entry fp32 NF4 code                        */
  int32_t blocksize;        /* 32, 64, 128 or 256                            */
  int32_t blocksize2;       /* nested: 256                                   */
  int32_t nested;           /* 1 = nested (double-quantized), 0 = plain;
                             * 2 = nested with the scale computed as ONE fused
                             * multiply-add, fmaf(code2[q], absmax2, offset): the
                             * contracted form a GPU build of nf4.py:36-39 may emit
                             * (solution/test_nf4_unpack.py:29-30 tolerates it), a
                             * debug form for the unpack only -- the fused GEMMs
                             * return NF4B_ERR_UNSUPPORTED for it */
  int32_t reserved;
} nf4b_qstate;

/* Unpack one packed NF4 tensor of `numel` values (numel/2 bytes, high nibble
 * first) into `out` (fp16 or fp32, numel values, row-major).
 * Replaces dequantize_nf4 (nf4.py:73-92).  */
int nf4b_dequant(const uint8_t* packed, const nf4b_qstate* qs, void* out, int32_t out_dtype,
                 int64_t numel, void* stream);

/* One unpack job of a batched sweep.  */
typedef struct nf4b_dequant_job {
  const uint8_t* packed;
  void* out;
  nf4b_qstate qs;
  int64_t numel;
  int32_t out_dtype;
  int32_t reserved;
} nf4b_dequant_job;

/* Size in bytes of the device-side plan nf4b_dequant_batched needs for n_jobs jobs.  */
int64_t nf4b_dequant_plan_bytes(int32_t n_jobs);

/* Build the device-side plan of a batched sweep: validates `jobs` (host array; a job of
 * numel 0 may have NULL pointers), copies them and the prefix sums of their work into
 * `plan_dev` (nf4b_dequant_plan_bytes(n_jobs) bytes of 16-byte aligned device memory owned
 * by the caller) with one cudaMemcpyAsync on `stream`, and returns the launch descriptor in
 * *launch (the CTA count in the low 32 bits, the kernel variant above them): pass it to
 * nf4b_dequant_batched unchanged.  The plan stays valid while the buffers it names do.
 * The plan also holds its launch's work counter (left zero by every launch), so launches of
 * one plan must not overlap: issue them on one stream.  At most 2^31 - 1 iterations of 2,048
 * values (NF4B_ERR_UNSUPPORTED beyond).  */
int nf4b_dequant_plan(const nf4b_dequant_job* jobs, int32_t n_jobs, void* plan_dev,
                      int64_t* launch, void* stream);

/* Unpack every job of a plan in ONE launch (replaces a loop of dequantize_nf4
 * calls, e.g. the 196 per-step unpacks of tools/bench_nf4.py:47).  `launch`: as returned by
 * nf4b_dequant_plan.  */
int nf4b_dequant_batched(const void* plan_dev, int32_t n_jobs, int64_t launch, void* stream);

/* Reads (and with reset != 0 clears) the device-side flag the unpack kernel sets when a
 * wait for one of its bulk copies ran out of time (the kernel then ends early instead of
 * hanging).  0 = no timeout since the last reset.  Synchronous.  No counterpart in the
 * reference.  */
int nf4b_dequant_error_flag(int* value, int reset);

/* LoRA adapter operands of a fused linear (peft lora.Linear, r = rank).
 * A is [rank, in] fp16 (lora_A.weight), B is [out, rank] fp16 (lora_B.weight),
 * scale = lora_alpha / r.  */
/* Adapter matrices and activations are read with 16-byte loads: a, b, xa and the dyb buffer
 * must be 16-byte aligned (NF4B_ERR_ALIGNMENT otherwise).  */
typedef struct nf4b_lora {
  const void* a;            /* fp16 [rank, in], contiguous                    */
  const void* b;            /* fp16 [out, rank], contiguous                   */
  float scale;
  int32_t rank;             /* 16                                             */
  void* xa;                 /* fwd: optional fp16 [n, rank] output of x A^T (saved for the backward) */
} nf4b_lora;

/* Y[n, out] = X[n, in] . W^T (+ bias) (+ (X A^T) B^T * scale), W the NF4 weight
 * [out, in] unpacked on the fly; fp16 in, fp32 accumulate, fp16 out.
 * Replaces the patched MatMul4Bit.forward (nf4.py:142-159).  */
int nf4b_linear_fwd(const void* x, const uint8_t* packed, const nf4b_qstate* qs,
                    const void* bias, const nf4b_lora* lora, void* y,
                    int64_t n, int64_t in_features, int64_t out_features, void* stream);

/* dX[n, in] = dY[n, out] . W (+ scale * (dY B) A), W re-unpacked on the fly.
 * Replaces bitsandbytes MatMul4Bit.backward's grad_A (nf4.py:131-133).
 * `dyb` (fp16 [n, rank]) receives dY . B when lora is given (needed by nf4b_lora_grads).  */
int nf4b_linear_bwd_dx(const void* dy, const uint8_t* packed, const nf4b_qstate* qs,
                       const nf4b_lora* lora, void* dyb, void* dx,
                       int64_t n, int64_t in_features, int64_t out_features, void* stream);

/* Split-K variants of the two above.  When a launch has fewer output tiles (128 weight
 * rows x 256 tokens) than the GPU has SMs, the K reduction of each tile is split over
 * several CTAs; the last CTA of a tile to finish adds the others' fp32 partials, so the
 * result differs from the unsplit call only in fp32 summation order.  Same arguments
 * as nf4b_linear_fwd / nf4b_linear_bwd_dx plus a caller-owned workspace:
 *   work        device buffer, 256-byte aligned, of at least
 *               nf4b_linear_work_bytes(n, in, out, backward) bytes (0 = no split for
 *               this shape on the current device: any pointer, or NULL, will do);
 *               its leading counter words must be zero before the first call and every
 *               call leaves them zero -- also one whose pipeline wait ran out (the last
 *               CTA to leave a launch clears them) -- so allocate it zeroed once and reuse it.
 *               Calls that may run concurrently (different streams) need distinct
 *               workspaces.  work == NULL runs unsplit.
 *   work_bytes  size of `work`; smaller than required -> NF4B_ERR_INVALID_ARG.
 * No counterpart in the reference, whose forward and backward are one cuBLAS GEMM each
 * (F.linear, nf4.py:152; bitsandbytes MatMul4Bit.backward).  */
int64_t nf4b_linear_work_bytes(int64_t n, int64_t in_features, int64_t out_features,
                               int32_t backward);
int nf4b_linear_fwd_ws(const void* x, const uint8_t* packed, const nf4b_qstate* qs,
                       const void* bias, const nf4b_lora* lora, void* y,
                       int64_t n, int64_t in_features, int64_t out_features,
                       void* work, int64_t work_bytes, void* stream);
int nf4b_linear_bwd_dx_ws(const void* dy, const uint8_t* packed, const nf4b_qstate* qs,
                          const nf4b_lora* lora, void* dyb, void* dx,
                          int64_t n, int64_t in_features, int64_t out_features,
                          void* work, int64_t work_bytes, void* stream);

/* Grouped forward: up to 3 NF4 weights that read the same activation X (q/k/v, gate/up) in
 * ONE launch; the tiles of all weights share the persistent grid, so small weights (k, v)
 * fill SMs the large one leaves idle and X streams through one pipeline.  Each item is one
 * nf4b_linear_fwd (its own output, bias, LoRA adapter and quant state); the split-K
 * workspace follows nf4b_linear_fwd_ws, sized by nf4b_linear_group_work_bytes over the
 * items' out_features.  No reference counterpart (the reference makes one F.linear call per
 * projection).  */
typedef struct nf4b_linear_item {
  const uint8_t* packed;     /* packed NF4 weight [out, in]                     */
  const nf4b_qstate* qs;
  const void* bias;          /* fp16 [out] or NULL                              */
  const nf4b_lora* lora;     /* or NULL                                         */
  void* y;                   /* fp16 [n, out]                                   */
  int64_t out_features;
} nf4b_linear_item;
int64_t nf4b_linear_group_work_bytes(int64_t n, int64_t in_features, const int64_t* out_features,
                                     int32_t n_items);
int nf4b_linear_fwd_group(const void* x, int64_t n, int64_t in_features,
                          const nf4b_linear_item* items, int32_t n_items, void* work,
                          int64_t work_bytes, void* stream);

/* Grouped backward: dX = sum_i dY_i . W_i (+ each item's LoRA dX term) for up to 3 NF4
 * weights that read the same input in the forward (q/k/v, gate/up) -- ONE GEMM whose K
 * dimension concatenates the items' out features, so the per-projection dX and their sum
 * never exist.  dx fp16 [n, in] is written (not accumulated).  Each item's dyb receives
 * dY_i . B_i when it has an adapter (for nf4b_lora_grads).  The split-K workspace follows
 * nf4b_linear_bwd_dx_ws, sized by nf4b_linear_bwd_group_work_bytes.  No reference
 * counterpart (autograd adds one dX per projection there).  */
typedef struct nf4b_linear_bwd_item {
  const void* dy;            /* fp16 [n, out] gradient of this projection's output */
  const uint8_t* packed;     /* packed NF4 weight [out, in]                     */
  const nf4b_qstate* qs;
  const nf4b_lora* lora;     /* or NULL                                         */
  void* dyb;                 /* fp16 [n, rank] when lora is given               */
  int64_t out_features;
} nf4b_linear_bwd_item;
int64_t nf4b_linear_bwd_group_work_bytes(int64_t n, int64_t in_features,
                                         const int64_t* out_features, int32_t n_items);
int nf4b_linear_bwd_dx_group(const nf4b_linear_bwd_item* items, int32_t n_items, void* dx,
                             int64_t n, int64_t in_features, void* work, int64_t work_bytes,
                             void* stream);

/* The gate/up projections of a SwiGLU MLP and the SwiGLU itself in ONE launch:
 *   gate_out[n, out] = X . Wg^T,  up_out[n, out] = X . Wu^T           (fp16, kept for the backward)
 *   m_out[n, out]    = fp16(gate_out * sigmoid(gate_out) * up_out)    (the input of down)
 * on the fp16 gate and up values, fp32 inside with one rounding and a fast exp and divide: the
 * rounding points of the reference's SwiGLU kernel (solution/swiglu.py:16-23, which its
 * unpad path calls, solution/unpad.py:60-63), and bit for bit what nf4b_swiglu_fwd gives.  Gate and up share the shape [out, in] (out a multiple of 64),
 * no bias, no adapter.  Each 128-row tile holds 64 features of both weights, so the epilogue
 * has gate and up of a feature side by side.  `work`: split-K workspace of
 * nf4b_linear_swiglu_work_bytes(n, in, out) bytes, same contract as nf4b_linear_fwd_ws.
 * No counterpart in the reference (there: two F.linear calls, then the SwiGLU kernel).  */
int64_t nf4b_linear_swiglu_work_bytes(int64_t n, int64_t in_features, int64_t out_features);
int nf4b_linear_fwd_swiglu(const void* x, int64_t n, int64_t in_features, const uint8_t* gate_packed,
                           const nf4b_qstate* gate_qs, const uint8_t* up_packed, const nf4b_qstate* up_qs,
                           void* gate_out, void* up_out, void* m_out, int64_t out_features, void* work,
                           int64_t work_bytes, void* stream);

/* The input gradient of a SwiGLU MLP's down projection with the SwiGLU backward in the same
 * launch: dm = fp16(dY . Wd) (Wd the NF4 down weight [out, in], in = the MLP width) is not
 * written; from it and the forward's gate and up [n, in] (fp16) the epilogue writes
 *   dup[n, in]   = fp16(dm * gate * sig)
 *   dgate[n, in] = fp16(dm * up * sig * (1 + gate * (1 - sig))),   sig = sigmoid(gate)
 * (nf4b_swiglu_bwd's arithmetic, bit for bit, on the dm nf4b_linear_bwd_dx_ws would write).
 * No adapter.  `work`: the split-K workspace of nf4b_linear_work_bytes(n, in, out, 1) bytes, same
 * contract as nf4b_linear_bwd_dx_ws.  No counterpart in the reference (there: dX of down, then
 * the SwiGLU backward kernel, solution/swiglu.py:26-37).  */
int nf4b_linear_bwd_dx_swiglu(const void* dy, const uint8_t* packed, const nf4b_qstate* qs, const void* gate,
                              const void* up, void* dgate, void* dup, int64_t n, int64_t in_features,
                              int64_t out_features, void* work, int64_t work_bytes, void* stream);

/* LoRA weight gradients (fp32 out, overwritten), both in one launch:
 *   dA[rank, in]  = scale * (dY B)^T X
 *   dB[out, rank] = scale * dY^T (X A^T)
 * x fp16 [n, in], dy fp16 [n, out], xa fp16 [n, rank], dyb fp16 [n, rank], all 16-byte
 * aligned; in and out multiples of 8.
 * `work`: caller-provided scratch of nf4b_lora_grads_work_bytes() bytes, 256-byte aligned (0
 * bytes: no token split, any pointer will do).  Its leading 4 KB are per-column-tile ticket
 * words that must be zero before the first call; every call leaves them zero, so allocate the
 * buffer zeroed once and reuse it (one per stream: calls that overlap on the GPU need distinct
 * buffers).  The sums are added in a fixed order: the result does not depend on scheduling.  */
int64_t nf4b_lora_grads_work_bytes(int64_t n, int64_t in_features, int64_t out_features, int32_t rank);
int nf4b_lora_grads(const void* x, const void* dy, const void* xa, const void* dyb, float scale,
                    float* da, float* db, void* work, int64_t n, int64_t in_features,
                    int64_t out_features, int32_t rank, void* stream);

/* The weight gradients of several adapters (e.g. q and v of one layer, whose backward runs at
 * the same time) in one launch.  Same math as nf4b_lora_grads per item; rank 16; at most 3
 * items.  `work`: scratch of nf4b_lora_grads_group_work_bytes(items, n_items, n) bytes (-1 for
 * invalid items) with the same ticket-word contract as nf4b_lora_grads.  */
typedef struct nf4b_lora_grads_item {
  const void* x;        /* fp16 [n, in_features], the projection's input        */
  const void* dy;       /* fp16 [n, out_features], the gradient of its output   */
  const void* xa;       /* fp16 [n, 16], x A^T from the forward                  */
  const void* dyb;      /* fp16 [n, 16], dY B from the backward dX GEMM          */
  float scale;          /* lora_alpha / r                                        */
  float* da;            /* fp32 [16, in_features] out                            */
  float* db;            /* fp32 [out_features, 16] out                           */
  int64_t in_features;
  int64_t out_features;
} nf4b_lora_grads_item;
int64_t nf4b_lora_grads_group_work_bytes(const nf4b_lora_grads_item* items, int32_t n_items, int64_t n);
int nf4b_lora_grads_group(const nf4b_lora_grads_item* items, int32_t n_items, void* work,
                          int64_t work_bytes, int64_t n, void* stream);

/* nf4b_lora_grads without the `work` argument, for callers that cannot call
 * cudaMalloc on this path (inside a framework that already holds the device's memory
 * in its own pool, or in a loop where allocating is not allowed).  It allocates
 * nothing: its split-token partial sums and ticket words live in a fixed device array of
 * NF4B_NOALLOC_SCRATCH_BYTES (4 MiB) inside the library, present on every GPU that loads the
 * library until the process exits.  A rank-16 problem needs at most ~2.4 MB of it (two 8 KB
 * partial tiles per SM plus 4 KB of tickets, whatever the shape and token count); a problem
 * that needed more (nf4b_lora_grads_work_bytes() > NF4B_NOALLOC_SCRATCH_BYTES) would return
 * NF4B_ERR_UNSUPPORTED with a message in nf4b_last_error().  All calls share the array, so
 * calls that overlap on the GPU race; the ticket words start zero and every call leaves them
 * zero, and each call writes every partial sum it reads.  The first call on a device looks up
 * the array's device address; make that first call before any stream capture.  The address is cached for the life of the process: after a
 * cudaDeviceReset (or a reset of the primary context) the library's module is loaded
 * again and this entry point must not be used on that device any more.  No counterpart in
 * the reference.  */
#define NF4B_NOALLOC_SCRATCH_BYTES (4 << 20)
int nf4b_lora_grads_noalloc(const void* x, const void* dy, const void* xa, const void* dyb,
                            float scale, float* da, float* db, int64_t n, int64_t in_features,
                            int64_t out_features, int32_t rank, void* stream);

/* Blockwise NF4 quantizer (the weight-loading side: what bitsandbytes.functional
 * .quantize_4bit produces, whose output nf4b_dequant unpacks).  w: fp16 or fp32 [numel]
 * (in_dtype NF4B_F16 / NF4B_F32), numel a multiple of blocksize (32 .. 4096, power of two).
 * Per block: absmax32[b] = max |x|; code = the number of NF4 midpoints <= x / absmax (nearest
 * code, a value on a midpoint takes the upper one); packed[numel/2], high nibble first.
 * nf4_mids: 15 fp32 midpoints of the 16-entry NF4 code, each the smallest fp32 >= the fp64
 * midpoint of its neighbours (so fp32 comparisons decide as fp64 ones).
 * Double quantization (absmax8 != NULL): offset[0] = fp32(mean of absmax32, summed in fp64
 * in a fixed order); per block of 256: absmax2 = max |absmax32 - offset|, absmax8 = the
 * number of code2_mids (255 midpoints of the 256-entry signed dynamic map) <= (absmax32 -
 * offset) / absmax2.  work: device scratch of nf4b_quantize_work_bytes() bytes.
 * All outputs are device buffers owned by the caller.  No reference counterpart in the
 * reference's own code (it calls bitsandbytes at model load).  */
int64_t nf4b_quantize_work_bytes(int64_t numel, int32_t blocksize);
int nf4b_quantize(const void* w, int32_t in_dtype, int64_t numel, int32_t blocksize,
                  const float* nf4_mids, const float* code2_mids, uint8_t* packed, float* absmax32,
                  uint8_t* absmax8, float* absmax2, float* offset, void* work, void* stream);

/* Reads (and with reset != 0 clears) the device-side flag the fused GEMMs set
 * when a pipeline wait ran out of time (the kernel then ends early instead of
 * hanging).  0 = no timeout since the last reset.  Synchronous.  */
int nf4b_gemm_error_flag(int* value, int reset);

/* Test hook for the split-K bookkeeping.  Arms a one-shot fault: the next fused-GEMM launch
 * of this process that splits K has work unit `unit` skip its ticket, as a K range that gave
 * up in its main loop would (that tile's output is then not written and the error flag reads
 * 4).  The launch still leaves the workspace's counters zero, so the call after it is correct.
 * No GPU fault is involved.  No counterpart in the reference.  */
int nf4b_test_drop_split_ticket(int32_t unit);

/* Launch geometry of the fused GEMMs on the current device: *sms = SMs (one persistent CTA
 * each), *pair_slots = 2-CTA clusters that can be resident at once (0 when the device runs
 * none; pairs of CTAs then never run).  Pairs tile 256 weight rows x 512 tokens, single CTAs
 * 128 rows x 256 (or 128) tokens; a cost model picks per launch.  The environment variable
 * STEW_NF4_PAIR overrides it: "0" single CTAs only, "1" pairs whenever pair_slots > 0, unset
 * or empty the cost model.  */
int nf4b_gemm_geometry(int* sms, int* pair_slots);

/* The CUDA error behind the last NF4B_ERR_CUDA returned on the calling host
 * thread ("<call>: <cudaErrorName> (<description>)"), or "" if none.  */
const char* nf4b_last_error(void);

/* Human-readable name of a status code.  */
const char* nf4b_status_string(int status);

/* Library build tag (for logs).  */
const char* nf4b_version(void);

#ifdef __cplusplus
}
#endif

#endif /* STEW_NF4_H */
