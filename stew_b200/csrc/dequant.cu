// Standalone NF4 unpack (sm_100a).
//
// Same arithmetic as the reference's `_nf4_unpack` (evilandangry/stew,
// solution/nf4.py:30-50):
//   nested: scale = code2[absmax8[blk]] * absmax2[blk / bs2] + offset  (nf4.py:36-39)
//   plain : scale = absmax[blk]                                        (nf4.py:41)
//   out[2j] = code[b >> 4] * scale, out[2j+1] = code[b & 15] * scale    (nf4.py:45-47)
// fp32 math with one rounding per operation (explicit __fmul_rn / __fadd_rn, so
// no FMA contraction can change a bit), one rounding to the output dtype.
//
// Work split (HBM-bound: 0.5 B in + 2 B out per value, ~1/64 B of scales):
//   one CTA = one chunk of 1024 packed 32-bit words (8192 values); thread t of
//   the CTA owns words t, t+256, t+512, t+768, so every warp-wide load reads
//   128 contiguous bytes and every warp-wide fp16 store writes 512 contiguous
//   bytes.  A 32-bit word is 8 values of one quantization block (blocks are
//   >= 32 values, word-aligned), so each word needs exactly one scale.
//   The 16-entry code sits in shared memory (16 distinct words in 16 banks: a
//   warp's lookups never conflict); the 256-entry second-level code is read
//   through the read-only cache.
// The batched variant runs many tensors in one launch: a device-side plan maps
// each CTA to (job, chunk).
#include <mutex>
#include <vector>

#include "common.cuh"

namespace nf4b {

constexpr int DQ_THREADS = 256;
constexpr int DQ_WORDS_PER_THREAD = 4;
constexpr int DQ_WORDS_PER_CTA = DQ_THREADS * DQ_WORDS_PER_THREAD;  // 1024 words = 8192 values

struct DqParams {
  const uint8_t* packed;
  void* out;
  const uint8_t* absmax8;
  const float* absmax32;
  const float* code2;
  const float* absmax2;
  const float* offset;
  const float* code;
  int64_t nwords;   // numel / 8
  int32_t log2_bs;  // log2(blocksize)
  int32_t log2_bs2; // log2(blocksize2)
  int32_t nested;
  int32_t f32out;
};

static_assert(sizeof(nf4b_dequant_job) % 8 == 0, "job struct layout");

__device__ __forceinline__ float block_scale(const DqParams& p, int64_t blk) {
  if (p.nested) {
    const uint32_t q = __ldg(p.absmax8 + blk);
    const float c2 = __ldg(p.code2 + q);
    const float a2 = __ldg(p.absmax2 + (blk >> p.log2_bs2));
    return __fadd_rn(__fmul_rn(c2, a2), __ldg(p.offset));
  }
  return __ldg(p.absmax32 + blk);
}

// Decode one packed word (bytes b0..b3 at increasing addresses, high nibble
// first) into 8 fp32 values in output order.
__device__ __forceinline__ void decode_word(uint32_t w, float scale, const float* s_code,
                                            float (&v)[8]) {
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint32_t byte = (w >> (8 * b)) & 0xFFu;
    v[2 * b] = __fmul_rn(s_code[byte >> 4], scale);
    v[2 * b + 1] = __fmul_rn(s_code[byte & 15u], scale);
  }
}

__device__ __forceinline__ void store_word(const DqParams& p, int64_t word, const float (&v)[8],
                                           bool aligned_out) {
  if (!p.f32out) {
    uint4 h;
    h.x = pack_half2(v[0], v[1]);
    h.y = pack_half2(v[2], v[3]);
    h.z = pack_half2(v[4], v[5]);
    h.w = pack_half2(v[6], v[7]);
    if (aligned_out) {
      st_cs_u128(static_cast<uint8_t*>(p.out) + word * 16, h);
    } else {
      uint32_t* o = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(p.out) + word * 16);
      // 4-byte aligned fallback (fp16 tensors are always 2-byte aligned; the host
      // routes anything not 4-byte aligned to the byte path below)
      o[0] = h.x; o[1] = h.y; o[2] = h.z; o[3] = h.w;
    }
  } else {
    float* o = reinterpret_cast<float*>(p.out) + word * 8;
    if (aligned_out) {
      st_cs_u128(o, make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]),
                               __float_as_uint(v[2]), __float_as_uint(v[3])));
      st_cs_u128(o + 4, make_uint4(__float_as_uint(v[4]), __float_as_uint(v[5]),
                                   __float_as_uint(v[6]), __float_as_uint(v[7])));
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = v[i];
    }
  }
}

// Processes chunk `chunk` (1024 words) of one tensor.  ALIGNED: packed is
// 4-byte aligned and out 16-byte aligned; otherwise byte loads and narrow stores.
template <bool ALIGNED>
__device__ __forceinline__ void dequant_chunk(const DqParams& p, int64_t chunk, const float* s_code) {
  const int64_t base = chunk * DQ_WORDS_PER_CTA + threadIdx.x;
  uint32_t w[DQ_WORDS_PER_THREAD];
#pragma unroll
  for (int j = 0; j < DQ_WORDS_PER_THREAD; ++j) {
    const int64_t word = base + int64_t(j) * DQ_THREADS;
    w[j] = 0;
    if (word < p.nwords) {
      if (ALIGNED) {
        w[j] = ld_nc_u32(p.packed + word * 4);
      } else {
        const uint8_t* b = p.packed + word * 4;
        w[j] = uint32_t(b[0]) | (uint32_t(b[1]) << 8) | (uint32_t(b[2]) << 16) |
               (uint32_t(b[3]) << 24);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < DQ_WORDS_PER_THREAD; ++j) {
    const int64_t word = base + int64_t(j) * DQ_THREADS;
    if (word < p.nwords) {
      const float scale = block_scale(p, (word << 3) >> p.log2_bs);
      float v[8];
      decode_word(w[j], scale, s_code, v);
      if (ALIGNED) {
        store_word(p, word, v, true);
      } else if (!p.f32out) {
        __half* o = static_cast<__half*>(p.out) + word * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = __float2half_rn(v[i]);
      } else {
        float* o = static_cast<float*>(p.out) + word * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = v[i];
      }
    }
  }
}

template <bool ALIGNED>
__global__ void __launch_bounds__(DQ_THREADS) nf4_dequant_kernel(const DqParams p) {
  __shared__ float s_code[16];
  if (threadIdx.x < 16) s_code[threadIdx.x] = __ldg(p.code + threadIdx.x);
  __syncthreads();
  dequant_chunk<ALIGNED>(p, blockIdx.x, s_code);
}

// Batched plan layout in device memory:
//   DqParams params[n_jobs]; int64_t cta_start[n_jobs + 1]
__global__ void __launch_bounds__(DQ_THREADS)
    nf4_dequant_batched_kernel(const DqParams* __restrict__ params,
                               const int64_t* __restrict__ cta_start, int32_t n_jobs) {
  __shared__ float s_code[16];
  __shared__ int s_job;
  const int64_t cta = blockIdx.x;
  if (threadIdx.x == 0) {
    int lo = 0, hi = n_jobs - 1;  // last job whose start <= cta
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (__ldg(cta_start + mid) <= cta) lo = mid; else hi = mid - 1;
    }
    s_job = lo;
  }
  __syncthreads();
  const int job = s_job;
  const DqParams& p = params[job];
  if (threadIdx.x < 16) s_code[threadIdx.x] = __ldg(p.code + threadIdx.x);
  __syncthreads();
  dequant_chunk<true>(p, cta - __ldg(cta_start + job), s_code);
}

// ------------------------------------------------------------------- host side
static int check_qstate(const nf4b_qstate* qs, int32_t* log2_bs, int32_t* log2_bs2) {
  NF4B_RETURN_IF(qs == nullptr || qs->code == nullptr, NF4B_ERR_INVALID_ARG);
  const int lb = ilog2_exact(qs->blocksize);
  NF4B_RETURN_IF(lb < 5 || lb > 8, NF4B_ERR_UNSUPPORTED);  // 32, 64, 128, 256 (nf4.py:66)
  *log2_bs = lb;
  *log2_bs2 = 0;
  if (qs->nested) {
    NF4B_RETURN_IF(!qs->absmax8 || !qs->code2 || !qs->absmax2 || !qs->offset,
                   NF4B_ERR_INVALID_ARG);
    NF4B_RETURN_IF(qs->blocksize2 != 256, NF4B_ERR_UNSUPPORTED);  // nf4.py:70
    *log2_bs2 = 8;
  } else {
    NF4B_RETURN_IF(!qs->absmax32, NF4B_ERR_INVALID_ARG);
  }
  return NF4B_OK;
}

static int make_params(const uint8_t* packed, const nf4b_qstate* qs, void* out, int32_t out_dtype,
                       int64_t numel, DqParams* p) {
  NF4B_RETURN_IF(packed == nullptr || out == nullptr, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(out_dtype != NF4B_F16 && out_dtype != NF4B_F32, NF4B_ERR_UNSUPPORTED);
  NF4B_RETURN_IF(numel < 0, NF4B_ERR_INVALID_ARG);
  int32_t lb = 0, lb2 = 0;
  int st = check_qstate(qs, &lb, &lb2);
  if (st != NF4B_OK) return st;
  NF4B_RETURN_IF(numel % qs->blocksize != 0, NF4B_ERR_UNSUPPORTED);  // nf4.py:69
  *p = DqParams{packed, out, qs->absmax8, qs->absmax32, qs->code2, qs->absmax2, qs->offset,
                qs->code, numel >> 3, lb, lb2, qs->nested ? 1 : 0, out_dtype == NF4B_F32};
  return NF4B_OK;
}

// Resolves the calling thread's device (the context current on the thread, as the
// caller's framework left it), makes sure that device's primary context is bound to
// this thread -- a thread can reach us with no current context (e.g. a worker thread
// whose framework-level device guard was a no-op), and driver-API calls such as the
// tensor-map encoder need one -- and checks for an sm_100 part.  Cached per thread.
int check_device() {
  static thread_local int cached_dev = -1;
  static thread_local int cached_ok = 0;
  int dev = 0;
  NF4B_CUDA_TRY(cudaGetDevice(&dev));
  if (dev != cached_dev) {
    NF4B_CUDA_TRY(cudaSetDevice(dev));
    int major = 0;
    NF4B_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    cached_dev = dev;
    cached_ok = (major == 10);
  }
  return cached_ok ? NF4B_OK : NF4B_ERR_DEVICE;
}

}  // namespace nf4b

using namespace nf4b;

extern "C" int nf4b_dequant(const uint8_t* packed, const nf4b_qstate* qs, void* out,
                            int32_t out_dtype, int64_t numel, void* stream) {
  DqParams p;
  int st = make_params(packed, qs, out, out_dtype, numel, &p);
  if (st != NF4B_OK) return st;
  if (numel == 0) return NF4B_OK;
  st = check_device();
  if (st != NF4B_OK) return st;
  const int64_t ctas = (p.nwords + DQ_WORDS_PER_CTA - 1) / DQ_WORDS_PER_CTA;
  NF4B_RETURN_IF(ctas > 0x7FFFFFFFll, NF4B_ERR_UNSUPPORTED);
  const bool al = aligned(packed, 4) && aligned(out, 16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (al)
    nf4_dequant_kernel<true><<<unsigned(ctas), DQ_THREADS, 0, s>>>(p);
  else
    nf4_dequant_kernel<false><<<unsigned(ctas), DQ_THREADS, 0, s>>>(p);
  return launch_status();
}

extern "C" int64_t nf4b_dequant_plan_bytes(int32_t n_jobs) {
  if (n_jobs <= 0) return 0;
  return int64_t(n_jobs) * int64_t(sizeof(DqParams)) + int64_t(n_jobs + 1) * 8;
}

extern "C" int nf4b_dequant_plan(const nf4b_dequant_job* jobs, int32_t n_jobs, void* plan_dev,
                                 int64_t* n_ctas, void* stream) {
  NF4B_RETURN_IF(jobs == nullptr || plan_dev == nullptr || n_ctas == nullptr || n_jobs <= 0,
                 NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(!aligned(plan_dev, 16), NF4B_ERR_ALIGNMENT);
  std::vector<uint8_t> host(size_t(nf4b_dequant_plan_bytes(n_jobs)));
  DqParams* params = reinterpret_cast<DqParams*>(host.data());
  int64_t* starts = reinterpret_cast<int64_t*>(host.data() + size_t(n_jobs) * sizeof(DqParams));
  int64_t total = 0;
  for (int i = 0; i < n_jobs; ++i) {
    int st = make_params(jobs[i].packed, &jobs[i].qs, jobs[i].out, jobs[i].out_dtype,
                         jobs[i].numel, &params[i]);
    if (st != NF4B_OK) return st;
    // the batched kernel has only the vectorised path
    NF4B_RETURN_IF(!aligned(jobs[i].packed, 4) || !aligned(jobs[i].out, 16), NF4B_ERR_ALIGNMENT);
    starts[i] = total;
    total += (params[i].nwords + DQ_WORDS_PER_CTA - 1) / DQ_WORDS_PER_CTA;
  }
  starts[n_jobs] = total;
  NF4B_RETURN_IF(total > 0x7FFFFFFFll, NF4B_ERR_UNSUPPORTED);
  *n_ctas = total;
  // A copy from pageable host memory returns once the source has been staged,
  // so the local buffer may be released right after.
  NF4B_CUDA_TRY(cudaMemcpyAsync(plan_dev, host.data(), host.size(), cudaMemcpyHostToDevice,
                                static_cast<cudaStream_t>(stream)));
  return NF4B_OK;
}

extern "C" int nf4b_dequant_batched(const void* plan_dev, int32_t n_jobs, int64_t n_ctas,
                                    void* stream) {
  NF4B_RETURN_IF(plan_dev == nullptr || n_jobs <= 0 || n_ctas < 0, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(n_ctas > 0x7FFFFFFFll, NF4B_ERR_UNSUPPORTED);
  if (n_ctas == 0) return NF4B_OK;
  int st = check_device();
  if (st != NF4B_OK) return st;
  const DqParams* params = static_cast<const DqParams*>(plan_dev);
  const int64_t* starts = reinterpret_cast<const int64_t*>(
      static_cast<const uint8_t*>(plan_dev) + size_t(n_jobs) * sizeof(DqParams));
  nf4_dequant_batched_kernel<<<unsigned(n_ctas), DQ_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      params, starts, n_jobs);
  return launch_status();
}
