// LoRA (rank 16) side kernels of the q/v adapter (peft lora.Linear,
// y = base(x) + lora_B(lora_A(x)) * scaling; the reference keeps peft's module and
// only touches its input cast, solution/rmsnorm.py:137-150).
//
//  lora_project16   out[t, r] = sum_k act[t, k] * W[r, k]       (X A^T forward, dY B backward)
//                   fp32 accumulate, fp16 result (what peft's fp16 autocast linear yields).
//                   HBM-bound on `act`; mma.sync tiles of 16 tokens, K split over 8 warps.
//  lora_outer16     G[r, c] = sum_t P[t, r] * Q[t, c]            (the two weight gradients)
//                   split over tokens; partial sums go to caller-provided scratch and a
//                   second kernel adds them up and applies the scale.
#include <mutex>

#include "common.cuh"

namespace nf4b {

// Rank-16 projection on the tensor cores (mma.sync m16n8k16, fp16 in, fp32 accumulate): a
// CTA of 8 warps owns 16 tokens, each warp one eighth of K; the eight partial 16x16 tiles are
// summed through shared memory.  Streams `act` once (HBM-bound); W (16 x K) stays in L2.
constexpr int LP_THREADS = 256;
constexpr int LP_WARPS = LP_THREADS / 32;
constexpr int LP_TOK = 16;

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// W(r, k) and W(r, k+1) as one half2 (k in the low half); k is even.
__device__ __forceinline__ uint32_t ld_w_pair(const __half* w, int64_t sr, int64_t sk, int r,
                                              int64_t k) {
  if (sk == 1) return __ldg(reinterpret_cast<const unsigned int*>(w + r * sr + k));
  const uint32_t lo = __ldg(reinterpret_cast<const unsigned short*>(w + r * sr + k * sk));
  const uint32_t hi = __ldg(reinterpret_cast<const unsigned short*>(w + r * sr + (k + 1) * sk));
  return lo | (hi << 16);
}

__global__ void __launch_bounds__(LP_THREADS)
    lora_project16_kernel(const __half* __restrict__ act, const __half* __restrict__ w, int64_t sr,
                          int64_t sk, __half* __restrict__ out, int64_t n, int64_t kdim) {
  __shared__ float red[LP_WARPS][LP_TOK][17];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;  // mma fragment coordinates
  const int64_t t0 = int64_t(blockIdx.x) * LP_TOK;
  const int64_t ksteps = kdim / 16;
  const int64_t per = (ksteps + LP_WARPS - 1) / LP_WARPS;
  const int64_t kb = warp * per;
  const int64_t ke = min64(ksteps, kb + per);
  const bool v0 = t0 + g < n, v1 = t0 + g + 8 < n;
  const unsigned int* x0 = reinterpret_cast<const unsigned int*>(act + (t0 + g) * kdim);
  const unsigned int* x1 = reinterpret_cast<const unsigned int*>(act + (t0 + g + 8) * kdim);
  float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
  for (int64_t ks = kb; ks < ke; ++ks) {
    const int64_t k = ks * 16 + 2 * c;
    uint32_t a[4];
    a[0] = v0 ? __ldg(x0 + (k >> 1)) : 0u;      // rows g / g+8, k..k+1
    a[1] = v1 ? __ldg(x1 + (k >> 1)) : 0u;
    a[2] = v0 ? __ldg(x0 + (k >> 1) + 4) : 0u;  // k+8..k+9
    a[3] = v1 ? __ldg(x1 + (k >> 1) + 4) : 0u;
    mma16816(d0, a, ld_w_pair(w, sr, sk, g, k), ld_w_pair(w, sr, sk, g, k + 8));
    mma16816(d1, a, ld_w_pair(w, sr, sk, 8 + g, k), ld_w_pair(w, sr, sk, 8 + g, k + 8));
  }
  red[warp][g][2 * c] = d0[0];
  red[warp][g][2 * c + 1] = d0[1];
  red[warp][g + 8][2 * c] = d0[2];
  red[warp][g + 8][2 * c + 1] = d0[3];
  red[warp][g][8 + 2 * c] = d1[0];
  red[warp][g][8 + 2 * c + 1] = d1[1];
  red[warp][g + 8][8 + 2 * c] = d1[2];
  red[warp][g + 8][8 + 2 * c + 1] = d1[3];
  __syncthreads();
  const int t = threadIdx.x >> 4, r = threadIdx.x & 15;
  float sum = 0.f;
#pragma unroll
  for (int ww = 0; ww < LP_WARPS; ++ww) sum += red[ww][t][r];
  if (t0 + t < n) out[(t0 + t) * 16 + r] = __float2half_rn(sum);
}

int lora_project16(const void* act, const void* w, int64_t w_stride_r, int64_t w_stride_k,
                   void* out, int64_t n, int64_t kdim, cudaStream_t s) {
  NF4B_RETURN_IF(kdim % 16 != 0, NF4B_ERR_UNSUPPORTED);
  NF4B_RETURN_IF(!aligned(act, 16) || !aligned(w, 4), NF4B_ERR_ALIGNMENT);
  if (n == 0) return NF4B_OK;
  const int64_t ctas = (n + LP_TOK - 1) / LP_TOK;
  NF4B_RETURN_IF(ctas > 0x7FFFFFFFll, NF4B_ERR_UNSUPPORTED);
  lora_project16_kernel<<<unsigned(ctas), LP_THREADS, 0, s>>>(
      static_cast<const __half*>(act), static_cast<const __half*>(w), w_stride_r, w_stride_k,
      static_cast<__half*>(out), n, kdim);
  return launch_status("lora_project16_kernel launch");
}

// ---------------------------------------------------------------- weight grads
constexpr int LO_THREADS = 128;
constexpr int LO_COLS = 2 * LO_THREADS;  // 256 columns per CTA
constexpr int LO_TSTAGE = 64;            // token rows of P staged per pass
constexpr int LO_TARGET_CTAS = 2 * 148;  // two waves' worth of CTAs on a 148-SM B200

static int64_t outer_splits(int64_t n, int64_t cols) {
  const int64_t col_ctas = (cols + LO_COLS - 1) / LO_COLS;
  int64_t s = (LO_TARGET_CTAS + col_ctas - 1) / col_ctas;
  const int64_t max_s = (n + LO_TSTAGE - 1) / LO_TSTAGE;
  if (s > max_s) s = max_s;
  return s < 1 ? 1 : s;
}

// partial[split][r][c] = sum over this split's tokens of P[t, r] * Q[t, c]
__global__ void __launch_bounds__(LO_THREADS)
    lora_outer16_kernel(const __half* __restrict__ P, const __half* __restrict__ Q, int64_t n,
                        int64_t cols, int64_t tok_per_split, float* __restrict__ partial) {
  __shared__ __align__(16) float ps[LO_TSTAGE * 16];
  const int64_t c = int64_t(blockIdx.x) * LO_COLS + 2 * threadIdx.x;
  const int64_t tb = int64_t(blockIdx.y) * tok_per_split;
  const int64_t te = min64(n, tb + tok_per_split);
  float acc[16][2];
#pragma unroll
  for (int r = 0; r < 16; ++r) acc[r][0] = acc[r][1] = 0.f;
  const bool cok = c < cols;  // cols is even
  for (int64_t ts = tb; ts < te; ts += LO_TSTAGE) {
    const int tl = int(min64(LO_TSTAGE, te - ts));
    __syncthreads();
    for (int e = threadIdx.x; e < tl * 16; e += LO_THREADS) ps[e] = __half2float(P[ts * 16 + e]);
    __syncthreads();
    if (cok) {
      // eight tokens' loads in flight before their multiply-adds
      constexpr int U = 8;
      int t = 0;
      for (; t < tl; t += U) {
        float2 q[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          q[u] = (t + u < tl) ? __half22float2(*reinterpret_cast<const __half2*>(Q + (ts + t + u) * cols + c))
                              : make_float2(0.f, 0.f);
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (t + u >= tl) break;  // rows past the staged ones hold stale values
          const float4* pr = reinterpret_cast<const float4*>(ps + (t + u) * 16);
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            const float4 p = pr[v4];
            acc[4 * v4 + 0][0] = fmaf(p.x, q[u].x, acc[4 * v4 + 0][0]);
            acc[4 * v4 + 0][1] = fmaf(p.x, q[u].y, acc[4 * v4 + 0][1]);
            acc[4 * v4 + 1][0] = fmaf(p.y, q[u].x, acc[4 * v4 + 1][0]);
            acc[4 * v4 + 1][1] = fmaf(p.y, q[u].y, acc[4 * v4 + 1][1]);
            acc[4 * v4 + 2][0] = fmaf(p.z, q[u].x, acc[4 * v4 + 2][0]);
            acc[4 * v4 + 2][1] = fmaf(p.z, q[u].y, acc[4 * v4 + 2][1]);
            acc[4 * v4 + 3][0] = fmaf(p.w, q[u].x, acc[4 * v4 + 3][0]);
            acc[4 * v4 + 3][1] = fmaf(p.w, q[u].y, acc[4 * v4 + 3][1]);
          }
        }
      }
    }
  }
  if (cok) {
    float* dst = partial + int64_t(blockIdx.y) * 16 * cols + c;
#pragma unroll
    for (int r = 0; r < 16; ++r)
      *reinterpret_cast<float2*>(dst + int64_t(r) * cols) = make_float2(acc[r][0], acc[r][1]);
  }
}

// out = scale * sum_s partial[s]; transpose_out: out[c][r] (dB [out, 16]) else out[r][c] (dA).
__global__ void lora_reduce_kernel(const float* __restrict__ partial, int64_t splits, int64_t cols,
                                   float scale, int transpose_out, float* __restrict__ out) {
  const int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;  // index into [16][cols]
  if (e >= 16 * cols) return;
  float sum = 0.f;
  for (int64_t s = 0; s < splits; ++s) sum += partial[s * 16 * cols + e];
  const int64_t r = e / cols, c = e - r * cols;
  if (transpose_out)
    out[c * 16 + r] = sum * scale;
  else
    out[e] = sum * scale;
}

static int outer_and_reduce(const __half* P, const __half* Q, int64_t n, int64_t cols, float scale,
                            int transpose_out, float* out, float* work, cudaStream_t s) {
  const int64_t splits = outer_splits(n, cols);
  const int64_t tps = (n + splits - 1) / splits;
  dim3 grid(unsigned((cols + LO_COLS - 1) / LO_COLS), unsigned(splits));
  lora_outer16_kernel<<<grid, LO_THREADS, 0, s>>>(P, Q, n, cols, tps, work);
  int st = launch_status();
  if (st != NF4B_OK) return st;
  const int64_t total = 16 * cols;
  lora_reduce_kernel<<<unsigned((total + 255) / 256), 256, 0, s>>>(work, splits, cols, scale,
                                                                  transpose_out, out);
  return launch_status();
}

}  // namespace nf4b

using namespace nf4b;

extern "C" int64_t nf4b_lora_grads_work_bytes(int64_t n, int64_t in_features, int64_t out_features,
                                              int32_t rank) {
  if (n < 0 || in_features <= 0 || out_features <= 0 || rank != 16) return -1;
  const int64_t a = outer_splits(n, in_features) * 16 * in_features;
  const int64_t b = outer_splits(n, out_features) * 16 * out_features;
  return (a > b ? a : b) * int64_t(sizeof(float));
}

extern "C" int nf4b_lora_grads(const void* x, const void* dy, const void* xa, const void* dyb,
                               float scale, float* da, float* db, void* work, int64_t n,
                               int64_t in_features, int64_t out_features, int32_t rank,
                               void* stream) {
  NF4B_RETURN_IF(!x || !dy || !xa || !dyb || !da || !db || !work, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(n < 0 || in_features <= 0 || out_features <= 0, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(rank != 16, NF4B_ERR_UNSUPPORTED);
  NF4B_RETURN_IF(in_features % 2 != 0 || out_features % 2 != 0, NF4B_ERR_UNSUPPORTED);
  NF4B_RETURN_IF(!aligned(x, 4) || !aligned(dy, 4) || !aligned(xa, 16) || !aligned(dyb, 16) ||
                     !aligned(work, 8),
                 NF4B_ERR_ALIGNMENT);
  int st = check_device();
  if (st != NF4B_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    NF4B_CUDA_TRY(cudaMemsetAsync(da, 0, size_t(16 * in_features) * sizeof(float), s));
    NF4B_CUDA_TRY(cudaMemsetAsync(db, 0, size_t(16 * out_features) * sizeof(float), s));
    return NF4B_OK;
  }
  // dA[r, i] = s * sum_t dyb[t, r] x[t, i]
  st = outer_and_reduce(static_cast<const __half*>(dyb), static_cast<const __half*>(x), n,
                        in_features, scale, 0, da, static_cast<float*>(work), s);
  if (st != NF4B_OK) return st;
  // dB[o, r] = s * sum_t dy[t, o] xa[t, r]  (computed as G[r, o], written transposed)
  return outer_and_reduce(static_cast<const __half*>(xa), static_cast<const __half*>(dy), n,
                          out_features, scale, 1, db, static_cast<float*>(work), s);
}

// ------------------------------------------------- entry point without allocation
// For callers that cannot call cudaMalloc on this path -- code running inside a framework that
// has already reserved the device's memory for its own pool (an allocation behind its back can
// fail or break its accounting), or a latency-critical loop where allocating is not allowed --
// nf4b_lora_grads_noalloc keeps its split-token partial sums in this fixed file-scope device
// array instead of a caller-provided buffer.  Every GPU that loads the library holds these
// NF4B_NOALLOC_SCRATCH_BYTES until the process exits.  All calls share it: calls that overlap on
// the GPU (other streams, other host threads) race on it.  Each call writes every partial sum it
// later reads, so nothing has to start at zero and no clearing is needed.
namespace nf4b {

static __device__ __align__(256) float g_lora_noalloc_scratch[NF4B_NOALLOC_SCRATCH_BYTES / sizeof(float)];

void record_message(const char* msg);  // capi.cu

// Device address of the scratch array for the calling thread's current device.  Host code must
// not hand the symbol itself to a kernel (on the host it names a host-side stand-in), so the
// address is looked up once per device, with that device current, and cached.
static int noalloc_scratch(float** out) {
  static std::mutex mu;
  static float* addr[64] = {nullptr};
  int dev = 0;
  NF4B_CUDA_TRY(cudaGetDevice(&dev));
  NF4B_RETURN_IF(dev < 0 || dev >= 64, NF4B_ERR_DEVICE);
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    NF4B_CUDA_TRY(cudaGetSymbolAddress(&p, g_lora_noalloc_scratch));
    addr[dev] = static_cast<float*>(p);
  }
  *out = addr[dev];
  return NF4B_OK;
}

}  // namespace nf4b

extern "C" int nf4b_lora_grads_noalloc(const void* x, const void* dy, const void* xa,
                                       const void* dyb, float scale, float* da, float* db,
                                       int64_t n, int64_t in_features, int64_t out_features,
                                       int32_t rank, void* stream) {
  NF4B_RETURN_IF(!x || !dy || !xa || !dyb || !da || !db, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(n < 0 || in_features <= 0 || out_features <= 0, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(rank != 16, NF4B_ERR_UNSUPPORTED);
  NF4B_RETURN_IF(in_features % 2 != 0 || out_features % 2 != 0, NF4B_ERR_UNSUPPORTED);
  NF4B_RETURN_IF(!aligned(x, 4) || !aligned(dy, 4) || !aligned(xa, 16) || !aligned(dyb, 16),
                 NF4B_ERR_ALIGNMENT);
  const int64_t need = nf4b_lora_grads_work_bytes(n, in_features, out_features, rank);
  if (need > int64_t(NF4B_NOALLOC_SCRATCH_BYTES)) {
    record_message("nf4b_lora_grads_noalloc: the split-token partial sums need more than "
                   "NF4B_NOALLOC_SCRATCH_BYTES; use nf4b_lora_grads with a caller buffer");
    return NF4B_ERR_UNSUPPORTED;
  }
  int st = check_device();
  if (st != NF4B_OK) return st;
  float* work = nullptr;
  st = noalloc_scratch(&work);
  if (st != NF4B_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    NF4B_CUDA_TRY(cudaMemsetAsync(da, 0, size_t(16 * in_features) * sizeof(float), s));
    NF4B_CUDA_TRY(cudaMemsetAsync(db, 0, size_t(16 * out_features) * sizeof(float), s));
    return NF4B_OK;
  }
  st = outer_and_reduce(static_cast<const __half*>(dyb), static_cast<const __half*>(x), n,
                        in_features, scale, 0, da, work, s);
  if (st != NF4B_OK) return st;
  return outer_and_reduce(static_cast<const __half*>(xa), static_cast<const __half*>(dy), n,
                          out_features, scale, 1, db, work, s);
}
