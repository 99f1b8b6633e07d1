// Elementwise and row-reduction kernels of the packed-token Qwen2 layer that surrounds the
// NF4 projections in the QLoRA step: RMSNorm (plain and fused with the residual add), rotary
// position embedding on q and k, and the SwiGLU product -- forward and backward.
//
// They replace the reference's Triton kernels of the same layer (solution/rmsnorm.py:19-50
// _rms_fwd/_rms_bwd, :152-190 _add_rms_fwd/_add_rms_bwd, solution/rope.py:24-52 rope_kernel,
// solution/swiglu.py:15-40) with the same rounding points:
//   RMSNorm      y = fp16(w * fp16(x * r)),  r = rsqrt(mean(x^2) + eps), fp32 math
//   add+RMSNorm  s = fp16(res + delta), then RMSNorm of s
//   RoPE         out[i] = x[i] c[i] - x[i+d] s[i],  out[i+d] = x[i+d] c[i+d] + x[i] s[i+d]
//                (the rotate-half convention of Qwen2); the backward applies the transpose
//   SwiGLU       m = fp16(g * sigmoid(g) * u), fp32 inside (solution/swiglu.py)
// All activations are fp16 row-major; one warp owns one row of a norm (16-byte loads, the
// row kept in registers between the two passes); the elementwise kernels move 16 bytes per
// thread and access.
#include "common.cuh"
#include "stew_step.h"

namespace nf4b {

// Two rows (one warp each) per 64-thread CTA: a ~1,300-row batch spreads over every SM.  The
// kernels are instantiated per row width (NC chunks of 256 features), so a row occupies only
// the registers it needs and many warps fit on an SM.
constexpr int NORM_WARPS = 2;
constexpr int NORM_MAX_CHUNKS = 16;   // 16 x 256 = 4096 features per row at most

__device__ __forceinline__ void h8_to_f(uint4 v, float (&f)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 f_to_h8(const float (&f)[8]) {
  uint4 v;
  uint32_t* p = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = pack_half2(f[2 * i], f[2 * i + 1]);
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float round_h(float v) { return __half2float(__float2half_rn(v)); }

// Forward RMSNorm of one row; `delta` (nullable) is added first (fused residual add) and the
// fp16 sum written to `sum`.
template <int NC>
__global__ void __launch_bounds__(32 * NORM_WARPS)
    rmsnorm_fwd_kernel(const __half* __restrict__ x, const __half* __restrict__ delta,
                       const float* __restrict__ w, float eps, __half* __restrict__ sum,
                       __half* __restrict__ y, float* __restrict__ rstd, int64_t rows) {
  grid_dep_wait();  // programmatic launch: no global access before the wait
  constexpr int hidden = NC * 256;
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * NORM_WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  constexpr int nc = NC;  // 256-value chunks: lane owns values [chunk*256 + lane*8, +8)
  const __half* xr = x + row * hidden;
  uint4 v[NC];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    if (c < nc) {
      const int off = c * 256 + lane * 8;
      v[c] = *reinterpret_cast<const uint4*>(xr + off);
      if (delta != nullptr) {
        float a[8], b[8];
        h8_to_f(v[c], a);
        h8_to_f(*reinterpret_cast<const uint4*>(delta + row * hidden + off), b);
#pragma unroll
        for (int i = 0; i < 8; ++i) a[i] = __fadd_rn(a[i], b[i]);
        v[c] = f_to_h8(a);  // the fp16 residual stream
        *reinterpret_cast<uint4*>(sum + row * hidden + off) = v[c];
      }
      float f[8];
      h8_to_f(v[c], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(f[i], f[i], ss);
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / float(hidden) + eps);
  if (lane == 0) rstd[row] = r;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    if (c < nc) {
      const int off = c * 256 + lane * 8;
      float f[8];
      h8_to_f(v[c], f);
      const float4 w0 = *reinterpret_cast<const float4*>(w + off);
      const float4 w1 = *reinterpret_cast<const float4*>(w + off + 4);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = __fmul_rn(wv[i], round_h(__fmul_rn(f[i], r)));
      *reinterpret_cast<uint4*>(y + row * hidden + off) = f_to_h8(f);
    }
  }
}

// Backward: dx = r * (w dy - xn * mean(w dy xn)) (+ dsum), xn = x r.
template <int NC>
__global__ void __launch_bounds__(32 * NORM_WARPS)
    rmsnorm_bwd_kernel(const __half* __restrict__ dy, const __half* __restrict__ x,
                       const float* __restrict__ w, const float* __restrict__ rstd,
                       const __half* __restrict__ dsum, __half* __restrict__ dx, int64_t rows) {
  grid_dep_wait();  // programmatic launch: no global access before the wait
  constexpr int hidden = NC * 256;
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * NORM_WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  constexpr int nc = NC;
  const float r = rstd[row];
  uint4 xv[NC], gv[NC];
  float dot = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    if (c < nc) {
      const int off = c * 256 + lane * 8;
      xv[c] = *reinterpret_cast<const uint4*>(x + row * hidden + off);
      gv[c] = *reinterpret_cast<const uint4*>(dy + row * hidden + off);
      float a[8], g[8];
      h8_to_f(xv[c], a);
      h8_to_f(gv[c], g);
      const float4 w0 = *reinterpret_cast<const float4*>(w + off);
      const float4 w1 = *reinterpret_cast<const float4*>(w + off + 4);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) dot = fmaf(wv[i] * g[i], a[i] * r, dot);
    }
  }
  const float cmean = warp_sum(dot) / float(hidden);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    if (c < nc) {
      const int off = c * 256 + lane * 8;
      float a[8], g[8], o[8];
      h8_to_f(xv[c], a);
      h8_to_f(gv[c], g);
      const float4 w0 = *reinterpret_cast<const float4*>(w + off);
      const float4 w1 = *reinterpret_cast<const float4*>(w + off + 4);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      float ds[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (dsum != nullptr) h8_to_f(*reinterpret_cast<const uint4*>(dsum + row * hidden + off), ds);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = r * (wv[i] * g[i] - a[i] * r * cmean) + ds[i];
      *reinterpret_cast<uint4*>(dx + row * hidden + off) = f_to_h8(o);
    }
  }
}

// RoPE on q [T, hq, D] and k [T, hk, D]: one thread per (token, head, 8 consecutive pairs).
// inverse = 1 applies the transposed rotation (the backward).
__global__ void rope_qk_kernel(const __half* __restrict__ q, const __half* __restrict__ k,
                               const float* __restrict__ cosv, const float* __restrict__ sinv,
                               __half* __restrict__ qo, __half* __restrict__ ko, int64_t tokens,
                               int hq, int hk, int head_dim, int inverse) {
  grid_dep_wait();  // programmatic launch: no global access before the wait
  const int d = head_dim >> 1;
  const int per_head = d >> 3;  // threads per (token, head)
  const int64_t per_tok = int64_t(hq + hk) * per_head;
  const int64_t tid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (tid >= tokens * per_tok) return;
  const int64_t t = tid / per_tok;
  const int rem = int(tid - t * per_tok);
  const int head = rem / per_head;
  const int i0 = (rem - head * per_head) * 8;
  const bool isq = head < hq;
  const __half* src = isq ? q + (t * hq + head) * head_dim : k + (t * hk + (head - hq)) * head_dim;
  __half* dst = isq ? qo + (t * hq + head) * head_dim : ko + (t * hk + (head - hq)) * head_dim;
  float a[8], b[8];
  h8_to_f(*reinterpret_cast<const uint4*>(src + i0), a);      // x[i]
  h8_to_f(*reinterpret_cast<const uint4*>(src + i0 + d), b);  // x[i+d]
  const float* cr = cosv + t * head_dim;
  const float* sr = sinv + t * head_dim;
  float oa[8], ob[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float c0 = cr[i0 + j], c1 = cr[i0 + d + j];
    const float s0 = sr[i0 + j], s1 = sr[i0 + d + j];
    if (!inverse) {
      oa[j] = __fsub_rn(__fmul_rn(a[j], c0), __fmul_rn(b[j], s0));
      ob[j] = __fadd_rn(__fmul_rn(b[j], c1), __fmul_rn(a[j], s1));
    } else {
      oa[j] = __fadd_rn(__fmul_rn(a[j], c0), __fmul_rn(b[j], s1));
      ob[j] = __fsub_rn(__fmul_rn(b[j], c1), __fmul_rn(a[j], s0));
    }
  }
  *reinterpret_cast<uint4*>(dst + i0) = f_to_h8(oa);
  *reinterpret_cast<uint4*>(dst + i0 + d) = f_to_h8(ob);
}

// sigmoid through the fast exp and divide (the reference's SwiGLU kernel, solution/swiglu.py,
// computes it in fp32 with Triton's fast exp as well); the fused gate/up GEMM's epilogue uses
// the same expression, so the two SwiGLU forwards agree bit for bit
__device__ __forceinline__ float sigmoid_fast(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// SwiGLU: 8 values per thread.
__global__ void swiglu_fwd_kernel(const __half* __restrict__ g, const __half* __restrict__ u,
                                  __half* __restrict__ m, int64_t n8) {
  grid_dep_wait();  // programmatic launch: no global access before the wait
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  float gf[8], uf[8], o[8];
  h8_to_f(reinterpret_cast<const uint4*>(g)[i], gf);
  h8_to_f(reinterpret_cast<const uint4*>(u)[i], uf);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = gf[j] * sigmoid_fast(gf[j]) * uf[j];
  reinterpret_cast<uint4*>(m)[i] = f_to_h8(o);
}

// du = fp16(dm g sig), dg = fp16(dm u sig (1 + g (1 - sig))), sig = sigmoid(g), all in fp32 with
// one rounding (the reference's backward, solution/swiglu.py:26-37).
__global__ void swiglu_bwd_kernel(const __half* __restrict__ dm, const __half* __restrict__ g,
                                  const __half* __restrict__ u, __half* __restrict__ dg,
                                  __half* __restrict__ du, int64_t n8) {
  grid_dep_wait();  // programmatic launch: no global access before the wait
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  float df[8], gf[8], uf[8], og[8], ou[8];
  h8_to_f(reinterpret_cast<const uint4*>(dm)[i], df);
  h8_to_f(reinterpret_cast<const uint4*>(g)[i], gf);
  h8_to_f(reinterpret_cast<const uint4*>(u)[i], uf);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float sg = sigmoid_fast(gf[j]);
    ou[j] = df[j] * gf[j] * sg;
    og[j] = df[j] * uf[j] * sg * (1.f + gf[j] * (1.f - sg));
  }
  reinterpret_cast<uint4*>(dg)[i] = f_to_h8(og);
  reinterpret_cast<uint4*>(du)[i] = f_to_h8(ou);
}

// ---------------------------------------------------------------- LM-head cross-entropy
// One CTA per row of fp16 logits [rows, vocab] (the counterpart of the reference's fused head
// loss, solution/head_loss.py: loss and, in a second pass over the row, the gradient
// softmax - onehot written in place over the logits).  Forward: each thread keeps an online
// maximum and sum of exponentials over its 8-wide vectors (online softmax, Milakov and
// Gimelshein 2018), the CTA merges the pairs, and loss = logsumexp - logit[label] in fp32.
constexpr int CE_THREADS = 512;

__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) {
    m = m2;
    s = s2;
    return;
  }
  if (m2 > m) {
    s = s * expf(m - m2) + s2;
    m = m2;
  } else {
    s = s + s2 * expf(m2 - m);
  }
}

__global__ void __launch_bounds__(CE_THREADS)
    ce_fwd_kernel(const __half* __restrict__ logits, const int64_t* __restrict__ labels,
                  float* __restrict__ loss, float* __restrict__ lse_out, int64_t vocab) {
  grid_dep_wait();  // programmatic launch: no global access before the wait
  const int64_t row = blockIdx.x;
  const __half* x = logits + row * vocab;
  float m = -INFINITY, s = 0.f;
  const int64_t nv = vocab >> 3;  // 8-wide vectors (rows are 16-byte aligned: vocab % 8 == 0)
  for (int64_t i = threadIdx.x; i < nv; i += CE_THREADS) {
    float f[8];
    h8_to_f(*reinterpret_cast<const uint4*>(x + 8 * i), f);
    float vm = f[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) vm = fmaxf(vm, f[j]);
    if (vm > m) {
      s = (m == -INFINITY) ? 0.f : s * expf(m - vm);
      m = vm;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) s += expf(f[j] - m);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    lse_merge(m, s, m2, s2);
  }
  __shared__ float sm[CE_THREADS / 32], ssum[CE_THREADS / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[warp] = m;
    ssum[warp] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = sm[0], st = ssum[0];
    for (int w = 1; w < CE_THREADS / 32; ++w) lse_merge(mm, st, sm[w], ssum[w]);
    const float lse = mm + logf(st);
    lse_out[row] = lse;
    const int64_t t = labels[row];
    loss[row] = (t < 0 || t >= vocab) ? 0.f : lse - __half2float(x[t]);
  }
}

// Backward, in place: logits[r, j] <- fp16(g * (exp(logits[r, j] - lse[r]) - [j == label[r]])),
// g = *gscale (the incoming gradient of the summed loss times a power-of-two scale that keeps
// the small probabilities of a 151,936-entry row out of fp16's subnormal range); rows whose
// label is outside [0, vocab) (ignored) get zeros.
__global__ void __launch_bounds__(CE_THREADS)
    ce_bwd_kernel(__half* __restrict__ logits, const int64_t* __restrict__ labels,
                  const float* __restrict__ lse_in, const float* __restrict__ gscale, int64_t vocab) {
  grid_dep_wait();  // programmatic launch: no global access before the wait
  const int64_t row = blockIdx.x;
  __half* x = logits + row * vocab;
  const int64_t t = labels[row];
  const bool ignored = t < 0 || t >= vocab;
  const float g = ignored ? 0.f : *gscale;
  const float lse = lse_in[row];
  const int64_t nv = vocab >> 3;
  for (int64_t i = threadIdx.x; i < nv; i += CE_THREADS) {
    float f[8];
    h8_to_f(*reinterpret_cast<const uint4*>(x + 8 * i), f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p = expf(f[j] - lse) - ((8 * i + j) == t ? 1.f : 0.f);
      f[j] = g * p;
    }
    *reinterpret_cast<uint4*>(x + 8 * i) = f_to_h8(f);
  }
}

static int norm_checks(int64_t rows, int64_t hidden) {
  NF4B_RETURN_IF(rows < 0 || hidden <= 0, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(hidden % 256 != 0 || hidden > 256 * NORM_MAX_CHUNKS, NF4B_ERR_UNSUPPORTED);
  return NF4B_OK;
}

static unsigned norm_grid(int64_t rows) { return unsigned((rows + NORM_WARPS - 1) / NORM_WARPS); }

}  // namespace nf4b

using namespace nf4b;

extern "C" int nf4b_rmsnorm_fwd(const void* x, const void* delta, const float* w, float eps,
                                void* sum, void* y, float* rstd, int64_t rows, int64_t hidden,
                                void* stream) {
  int st = norm_checks(rows, hidden);
  if (st != NF4B_OK) return st;
  NF4B_RETURN_IF(!x || !w || !y || !rstd || (delta && !sum), NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(!aligned(x, 16) || !aligned(w, 16) || !aligned(y, 16) ||
                     (delta && (!aligned(delta, 16) || !aligned(sum, 16))),
                 NF4B_ERR_ALIGNMENT);
  if (rows == 0) return NF4B_OK;
  st = check_device();
  if (st != NF4B_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __half* xh = static_cast<const __half*>(x);
  const __half* dh = static_cast<const __half*>(delta);
  __half* sh = static_cast<__half*>(sum);
  __half* yh = static_cast<__half*>(y);
  switch (hidden >> 8) {
#define NF4B_NORM_FWD(NC_)                                                                     \
  case NC_:                                                                                    \
    NF4B_CUDA_TRY(launch_pdl(rmsnorm_fwd_kernel<NC_>, dim3(norm_grid(rows)), dim3(32 * NORM_WARPS), \
                             size_t(0), s, xh, dh, w, eps, sh, yh, rstd, rows));              \
    break;
    NF4B_NORM_FWD(1) NF4B_NORM_FWD(2) NF4B_NORM_FWD(3) NF4B_NORM_FWD(4) NF4B_NORM_FWD(5)
    NF4B_NORM_FWD(6) NF4B_NORM_FWD(7) NF4B_NORM_FWD(8) NF4B_NORM_FWD(9) NF4B_NORM_FWD(10)
    NF4B_NORM_FWD(11) NF4B_NORM_FWD(12) NF4B_NORM_FWD(13) NF4B_NORM_FWD(14) NF4B_NORM_FWD(15)
    NF4B_NORM_FWD(16)
#undef NF4B_NORM_FWD
    default:
      return NF4B_ERR_UNSUPPORTED;
  }
  return launch_status("rmsnorm_fwd_kernel launch");
}

extern "C" int nf4b_rmsnorm_bwd(const void* dy, const void* x, const float* w, const float* rstd,
                                const void* dsum, void* dx, int64_t rows, int64_t hidden,
                                void* stream) {
  int st = norm_checks(rows, hidden);
  if (st != NF4B_OK) return st;
  NF4B_RETURN_IF(!dy || !x || !w || !rstd || !dx, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(!aligned(dy, 16) || !aligned(x, 16) || !aligned(w, 16) || !aligned(dx, 16) ||
                     (dsum && !aligned(dsum, 16)),
                 NF4B_ERR_ALIGNMENT);
  if (rows == 0) return NF4B_OK;
  st = check_device();
  if (st != NF4B_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __half* gh = static_cast<const __half*>(dy);
  const __half* xh = static_cast<const __half*>(x);
  const __half* dsh = static_cast<const __half*>(dsum);
  __half* dxh = static_cast<__half*>(dx);
  switch (hidden >> 8) {
#define NF4B_NORM_BWD(NC_)                                                                     \
  case NC_:                                                                                    \
    NF4B_CUDA_TRY(launch_pdl(rmsnorm_bwd_kernel<NC_>, dim3(norm_grid(rows)), dim3(32 * NORM_WARPS), \
                             size_t(0), s, gh, xh, w, rstd, dsh, dxh, rows));                 \
    break;
    NF4B_NORM_BWD(1) NF4B_NORM_BWD(2) NF4B_NORM_BWD(3) NF4B_NORM_BWD(4) NF4B_NORM_BWD(5)
    NF4B_NORM_BWD(6) NF4B_NORM_BWD(7) NF4B_NORM_BWD(8) NF4B_NORM_BWD(9) NF4B_NORM_BWD(10)
    NF4B_NORM_BWD(11) NF4B_NORM_BWD(12) NF4B_NORM_BWD(13) NF4B_NORM_BWD(14) NF4B_NORM_BWD(15)
    NF4B_NORM_BWD(16)
#undef NF4B_NORM_BWD
    default:
      return NF4B_ERR_UNSUPPORTED;
  }
  return launch_status("rmsnorm_bwd_kernel launch");
}

extern "C" int nf4b_rope_qk(const void* q, const void* k, const float* cos_t, const float* sin_t,
                            void* q_out, void* k_out, int64_t tokens, int32_t q_heads,
                            int32_t k_heads, int32_t head_dim, int32_t inverse, void* stream) {
  NF4B_RETURN_IF(tokens < 0 || q_heads < 0 || k_heads < 0 || head_dim <= 0, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(head_dim % 16 != 0, NF4B_ERR_UNSUPPORTED);
  NF4B_RETURN_IF((q_heads && (!q || !q_out)) || (k_heads && (!k || !k_out)) || !cos_t || !sin_t,
                 NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF((q && !aligned(q, 16)) || (k && !aligned(k, 16)) || (q_out && !aligned(q_out, 16)) ||
                     (k_out && !aligned(k_out, 16)),
                 NF4B_ERR_ALIGNMENT);
  const int64_t threads = tokens * (q_heads + k_heads) * (head_dim / 16);
  if (threads == 0) return NF4B_OK;
  int st = check_device();
  if (st != NF4B_OK) return st;
  NF4B_CUDA_TRY(launch_pdl(rope_qk_kernel, dim3(unsigned((threads + 255) / 256)), dim3(256),
                           size_t(0), static_cast<cudaStream_t>(stream),
                           static_cast<const __half*>(q), static_cast<const __half*>(k), cos_t,
                           sin_t, static_cast<__half*>(q_out), static_cast<__half*>(k_out), tokens,
                           q_heads, k_heads, head_dim, inverse));
  return launch_status("rope_qk_kernel launch");
}

extern "C" int nf4b_swiglu_fwd(const void* gate, const void* up, void* out, int64_t n, void* stream) {
  NF4B_RETURN_IF(n < 0 || (n > 0 && (!gate || !up || !out)), NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(n % 8 != 0, NF4B_ERR_UNSUPPORTED);
  NF4B_RETURN_IF(!aligned(gate, 16) || !aligned(up, 16) || !aligned(out, 16), NF4B_ERR_ALIGNMENT);
  if (n == 0) return NF4B_OK;
  int st = check_device();
  if (st != NF4B_OK) return st;
  const int64_t n8 = n / 8;
  NF4B_CUDA_TRY(launch_pdl(swiglu_fwd_kernel, dim3(unsigned((n8 + 255) / 256)), dim3(256),
                           size_t(0), static_cast<cudaStream_t>(stream),
                           static_cast<const __half*>(gate), static_cast<const __half*>(up),
                           static_cast<__half*>(out), n8));
  return launch_status("swiglu_fwd_kernel launch");
}

extern "C" int nf4b_swiglu_bwd(const void* dout, const void* gate, const void* up, void* dgate,
                               void* dup, int64_t n, void* stream) {
  NF4B_RETURN_IF(n < 0 || (n > 0 && (!dout || !gate || !up || !dgate || !dup)), NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(n % 8 != 0, NF4B_ERR_UNSUPPORTED);
  NF4B_RETURN_IF(!aligned(dout, 16) || !aligned(gate, 16) || !aligned(up, 16) || !aligned(dgate, 16) ||
                     !aligned(dup, 16),
                 NF4B_ERR_ALIGNMENT);
  if (n == 0) return NF4B_OK;
  int st = check_device();
  if (st != NF4B_OK) return st;
  const int64_t n8 = n / 8;
  NF4B_CUDA_TRY(launch_pdl(swiglu_bwd_kernel, dim3(unsigned((n8 + 255) / 256)), dim3(256),
                           size_t(0), static_cast<cudaStream_t>(stream),
                           static_cast<const __half*>(dout), static_cast<const __half*>(gate),
                           static_cast<const __half*>(up), static_cast<__half*>(dgate),
                           static_cast<__half*>(dup), n8));
  return launch_status("swiglu_bwd_kernel launch");
}

extern "C" int nf4b_ce_fwd(const void* logits, const int64_t* labels, float* loss, float* lse,
                           int64_t rows, int64_t vocab, void* stream) {
  NF4B_RETURN_IF(rows < 0 || vocab <= 0, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(rows > 0 && (!logits || !labels || !loss || !lse), NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(vocab % 8 != 0 || rows > 0x7FFFFFFFll, NF4B_ERR_UNSUPPORTED);
  NF4B_RETURN_IF(!aligned(logits, 16), NF4B_ERR_ALIGNMENT);
  if (rows == 0) return NF4B_OK;
  int st = check_device();
  if (st != NF4B_OK) return st;
  NF4B_CUDA_TRY(launch_pdl(ce_fwd_kernel, dim3(unsigned(rows)), dim3(CE_THREADS), size_t(0),
                           static_cast<cudaStream_t>(stream), static_cast<const __half*>(logits),
                           labels, loss, lse, vocab));
  return launch_status("ce_fwd_kernel launch");
}

extern "C" int nf4b_ce_bwd(void* logits, const int64_t* labels, const float* lse, const float* gscale,
                           int64_t rows, int64_t vocab, void* stream) {
  NF4B_RETURN_IF(rows < 0 || vocab <= 0, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(rows > 0 && (!logits || !labels || !lse || !gscale), NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(vocab % 8 != 0 || rows > 0x7FFFFFFFll, NF4B_ERR_UNSUPPORTED);
  NF4B_RETURN_IF(!aligned(logits, 16), NF4B_ERR_ALIGNMENT);
  if (rows == 0) return NF4B_OK;
  int st = check_device();
  if (st != NF4B_OK) return st;
  NF4B_CUDA_TRY(launch_pdl(ce_bwd_kernel, dim3(unsigned(rows)), dim3(CE_THREADS), size_t(0),
                           static_cast<cudaStream_t>(stream), static_cast<__half*>(logits), labels,
                           lse, gscale, vocab));
  return launch_status("ce_bwd_kernel launch");
}
