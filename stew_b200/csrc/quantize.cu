// Blockwise NF4 quantizer with double quantization of the block scales -- the weight-loading
// side of the path (what bitsandbytes.functional.quantize_4bit produces for the reference,
// which calls it at model load; the unpack in dequant.cu is its inverse).
//
//   level 1 (nf4_quantize_kernel): per block of `blocksize` values, absmax = max |x| (fp32),
//            normed = x / absmax (fp32), code index = the number of NF4 midpoints <= normed
//            (nearest code; a value on a midpoint takes the upper code), two indices per byte,
//            high nibble first.
//   mean     (absmax_mean_kernel): the mean of the block absmax values, summed in fp64 in a
//            fixed order (per-CTA partials, then one CTA) and rounded once to fp32: the offset.
//   level 2 (absmax_quantize_kernel): per block of 256 absmax values, centred = absmax - offset,
//            absmax2 = max |centred|, code = the number of signed-dynamic-map midpoints <=
//            centred / absmax2.
// Midpoints of adjacent codes are taken in fp64 and passed as the smallest fp32 value >= each
// midpoint, so an fp32 comparison `v >= mid` decides exactly as the fp64 one would.
#include "common.cuh"

namespace nf4b {

constexpr int QZ_WARPS = 8;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float load_f(const void* p, int dtype, int64_t i) {
  return dtype == NF4B_F32 ? static_cast<const float*>(p)[i] : __half2float(static_cast<const __half*>(p)[i]);
}

// One warp per block; lane l handles the byte pairs l, l+32, ... of the block.
__global__ void __launch_bounds__(32 * QZ_WARPS)
    nf4_quantize_kernel(const void* __restrict__ w, int dtype, int64_t nblocks, int blocksize,
                        const float* __restrict__ mids, uint8_t* __restrict__ packed,
                        float* __restrict__ absmax) {
  __shared__ float s_mid[15];
  if (threadIdx.x < 15) s_mid[threadIdx.x] = mids[threadIdx.x];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t blk = int64_t(blockIdx.x) * QZ_WARPS + (threadIdx.x >> 5);
  if (blk >= nblocks) return;
  const int64_t base = blk * blocksize;
  const int pairs = blocksize / 2;
  float m = 0.f;
  for (int p = lane; p < pairs; p += 32)
    m = fmaxf(m, fmaxf(fabsf(load_f(w, dtype, base + 2 * p)), fabsf(load_f(w, dtype, base + 2 * p + 1))));
  m = warp_max(m);
  if (lane == 0) absmax[blk] = m;
  const float denom = m == 0.f ? 1.f : m;
  for (int p = lane; p < pairs; p += 32) {
    uint32_t idx[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float v = __fdiv_rn(load_f(w, dtype, base + 2 * p + e), denom);
      uint32_t c = 0;
#pragma unroll
      for (int i = 0; i < 15; ++i) c += v >= s_mid[i] ? 1u : 0u;
      idx[e] = c;
    }
    packed[base / 2 + p] = uint8_t((idx[0] << 4) | idx[1]);
  }
}

constexpr int QM_THREADS = 256;

// Partial fp64 sums of absmax over contiguous ranges, one per CTA, summed in a fixed order.
__global__ void __launch_bounds__(QM_THREADS)
    absmax_mean_kernel(const float* __restrict__ absmax, int64_t n, int64_t per_cta,
                       double* __restrict__ partial) {
  __shared__ double red[QM_THREADS];
  const int64_t b = int64_t(blockIdx.x) * per_cta;
  const int64_t e = min64(n, b + per_cta);
  double s = 0.0;
  for (int64_t i = b + threadIdx.x; i < e; i += QM_THREADS) s += double(absmax[i]);
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = QM_THREADS / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) partial[blockIdx.x] = red[0];
}

__global__ void __launch_bounds__(QM_THREADS)
    absmax_mean_final_kernel(const double* __restrict__ partial, int64_t parts, int64_t n,
                             float* __restrict__ offset) {
  __shared__ double red[QM_THREADS];
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < parts; i += QM_THREADS) s += partial[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = QM_THREADS / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) *offset = float(red[0] / double(n));
}

// One warp per 256 absmax values (8 per lane); binary search over the 255 midpoints.
__global__ void __launch_bounds__(32 * QZ_WARPS)
    absmax_quantize_kernel(const float* __restrict__ absmax, int64_t n, const float* __restrict__ offset,
                           const float* __restrict__ mids, uint8_t* __restrict__ absmax8,
                           float* __restrict__ absmax2) {
  __shared__ float s_mid[255];
  for (int i = threadIdx.x; i < 255; i += blockDim.x) s_mid[i] = mids[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t blk = int64_t(blockIdx.x) * QZ_WARPS + (threadIdx.x >> 5);
  if (blk * 256 >= n) return;
  const float off = *offset;
  float c[8];
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int64_t i = blk * 256 + lane + 32 * j;
    c[j] = i < n ? __fsub_rn(absmax[i], off) : 0.f;
    m = fmaxf(m, fabsf(c[j]));
  }
  m = warp_max(m);
  if (lane == 0) absmax2[blk] = m;
  const float denom = m == 0.f ? 1.f : m;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int64_t i = blk * 256 + lane + 32 * j;
    if (i >= n) continue;
    const float v = __fdiv_rn(c[j], denom);
    int lo = 0, hi = 255;  // number of midpoints <= v, in [0, 255]
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (v >= s_mid[mid])
        lo = mid + 1;
      else
        hi = mid;
    }
    absmax8[i] = uint8_t(lo);
  }
}

}  // namespace nf4b

using namespace nf4b;

extern "C" int64_t nf4b_quantize_work_bytes(int64_t numel, int32_t blocksize) {
  if (numel <= 0 || blocksize <= 0) return 0;
  const int64_t nb = numel / blocksize;
  const int64_t parts = (nb + 4095) / 4096;
  return 16 + parts * int64_t(sizeof(double));
}

extern "C" int nf4b_quantize(const void* w, int32_t in_dtype, int64_t numel, int32_t blocksize,
                             const float* nf4_mids, const float* code2_mids, uint8_t* packed,
                             float* absmax32, uint8_t* absmax8, float* absmax2, float* offset,
                             void* work, void* stream) {
  NF4B_RETURN_IF(!w || !nf4_mids || !packed || !absmax32, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(numel < 0, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(in_dtype != NF4B_F16 && in_dtype != NF4B_F32, NF4B_ERR_UNSUPPORTED);
  NF4B_RETURN_IF(ilog2_exact(blocksize) < 5 || blocksize > 4096, NF4B_ERR_UNSUPPORTED);
  NF4B_RETURN_IF(numel % blocksize != 0, NF4B_ERR_UNSUPPORTED);
  const bool nested = absmax8 != nullptr;
  NF4B_RETURN_IF(nested && (!code2_mids || !absmax2 || !offset || !work), NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(nested && !aligned(work, 8), NF4B_ERR_ALIGNMENT);
  if (numel == 0) return NF4B_OK;
  int st = check_device();
  if (st != NF4B_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t nb = numel / blocksize;
  nf4_quantize_kernel<<<unsigned((nb + QZ_WARPS - 1) / QZ_WARPS), 32 * QZ_WARPS, 0, s>>>(
      w, in_dtype, nb, blocksize, nf4_mids, packed, absmax32);
  st = launch_status("nf4_quantize_kernel launch");
  if (st != NF4B_OK || !nested) return st;
  const int64_t per = 4096;
  const int64_t parts = (nb + per - 1) / per;
  double* partial = reinterpret_cast<double*>(static_cast<uint8_t*>(work) + 16);
  absmax_mean_kernel<<<unsigned(parts), QM_THREADS, 0, s>>>(absmax32, nb, per, partial);
  st = launch_status("absmax_mean_kernel launch");
  if (st != NF4B_OK) return st;
  absmax_mean_final_kernel<<<1, QM_THREADS, 0, s>>>(partial, parts, nb, offset);
  st = launch_status("absmax_mean_final_kernel launch");
  if (st != NF4B_OK) return st;
  const int64_t nb2 = (nb + 255) / 256;
  absmax_quantize_kernel<<<unsigned((nb2 + QZ_WARPS - 1) / QZ_WARPS), 32 * QZ_WARPS, 0, s>>>(
      absmax32, nb, offset, code2_mids, absmax8, absmax2);
  return launch_status("absmax_quantize_kernel launch");
}
