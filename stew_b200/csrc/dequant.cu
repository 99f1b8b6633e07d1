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
// General path (fp32 out, unaligned buffers, numel not a multiple of 64), HBM-bound:
//   one CTA = one chunk of 1024 packed 32-bit words (8192 values); thread t of
//   the CTA owns words t, t+256, t+512, t+768, so every warp-wide load reads
//   128 contiguous bytes and every warp-wide fp16 store writes 512 contiguous
//   bytes.  A 32-bit word is 8 values of one quantization block (blocks are
//   >= 32 values, word-aligned), so each word needs exactly one scale.
//   The 16-entry code sits in shared memory (16 distinct words in 16 banks: a
//   warp's lookups never conflict); the 256-entry second-level code is read
//   through the read-only cache.
// The main fp16 path is the chunk kernel further down; its batched variant runs many
// tensors in one launch from a device-side plan.
#include <mutex>
#include <vector>

#include <cstdlib>

#include "common.cuh"
#include "nf4_decode.cuh"

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

// ---------------------------------------------------------------- chunk kernel
// Main path (fp16 out, 16-byte aligned buffers, numel a multiple of 64): one lane owns one
// 64-value chunk (32 packed bytes, one scale for blocksize >= 64, two for 32), builds the
// block's 16-entry fp16 table in registers (nf4_decode.cuh: T[i] = fp16(code[i] * scale),
// bit-identical to the reference's per-value multiply-then-round) and decodes 8 words with
// byte permutes.  The warp's 32 chunks (4 KB of fp16) go through a per-warp shared buffer,
// written with the 16-byte slot XOR-swizzled by (lane & 7) and read back transposed, so both
// sides are bank-conflict free and every global store instruction writes 512 contiguous
// bytes.  Persistent grid: warps stride over 32-chunk iterations; in the batched kernel a
// warp's iterations ascend, so its job index only moves forward.
constexpr int DQ2_THREADS = 256;
constexpr int DQ2_WARPS = DQ2_THREADS / 32;
constexpr int DQ2_CHUNKS_PER_ITER = 32;  // one per lane
constexpr int DQ2_CTAS_PER_SM = 3;       // persistent grid: 24 resident warps per SM

__device__ __forceinline__ void load_code16(const float* code, float (&c)[16]) {
  const float4* c4 = reinterpret_cast<const float4*>(code);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 v = __ldg(c4 + i);
    c[4 * i] = v.x; c[4 * i + 1] = v.y; c[4 * i + 2] = v.z; c[4 * i + 3] = v.w;
  }
}

// One warp iteration: chunks [iter*32, iter*32+32) of job p.
__device__ __forceinline__ void dequant_iter_v2(const DqParams& p, int64_t nchunks, int64_t iter,
                                                const float (&code)[16], uint8_t* wbuf) {
  const int lane = threadIdx.x & 31;
  const int64_t ch = iter * DQ2_CHUNKS_PER_ITER + lane;
  const bool valid = ch < nchunks;
  uint4 w0 = make_uint4(0, 0, 0, 0), w1 = w0;
  float s0 = 0.f, s1 = 0.f;
  if (valid) {
    const uint4* src = reinterpret_cast<const uint4*>(p.packed + ch * 32);
    w0 = __ldg(src);
    w1 = __ldg(src + 1);
    if (p.log2_bs >= 6) {
      const int64_t blk = (ch << 6) >> p.log2_bs;
      s0 = s1 = block_scale(p, blk);
    } else {  // 32-value blocks: two per chunk
      s0 = block_scale(p, 2 * ch);
      s1 = block_scale(p, 2 * ch + 1);
    }
  }
  const Nf4Table t0 = make_table(code, s0);
  const Nf4Table t1 = (p.log2_bs >= 6) ? t0 : make_table(code, s1);
  const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  const uint32_t row = smem_u32(wbuf) + uint32_t(lane) * 128u;
  const uint32_t key = uint32_t(lane & 7);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint4 v = decode_word_f16(j < 4 ? t0 : t1, w[j]);
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(row + ((uint32_t(j) ^ key) << 4)),
                 "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
  }
  __syncwarp();
  uint8_t* out = static_cast<uint8_t*>(p.out) + iter * (DQ2_CHUNKS_PER_ITER * 128);
  const int c = lane & 7;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int b = 4 * r + (lane >> 3);  // chunk of this 16-byte piece
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_u32(wbuf) + uint32_t(b) * 128u + ((uint32_t(c) ^ uint32_t(b & 7)) << 4)));
    if (iter * DQ2_CHUNKS_PER_ITER + b < nchunks) st_cs_u128(out + r * 512 + lane * 16, v);
  }
  __syncwarp();
}

__global__ void __launch_bounds__(DQ2_THREADS, DQ2_CTAS_PER_SM) nf4_dequant_chunk_kernel(const DqParams p) {
  __shared__ __align__(128) uint8_t stage[DQ2_WARPS][4096];
  const int warp = threadIdx.x >> 5;
  float code[16];
  load_code16(p.code, code);
  const int64_t nchunks = p.nwords >> 3;
  const int64_t iters = (nchunks + DQ2_CHUNKS_PER_ITER - 1) / DQ2_CHUNKS_PER_ITER;
  for (int64_t it = int64_t(blockIdx.x) * DQ2_WARPS + warp; it < iters;
       it += int64_t(gridDim.x) * DQ2_WARPS)
    dequant_iter_v2(p, nchunks, it, code, stage[warp]);
}

// Batched plan in device memory: DqParams params[n_jobs]; int64_t iter_start[n_jobs + 1]
// (prefix sums of 32-chunk iterations).
__global__ void __launch_bounds__(DQ2_THREADS, DQ2_CTAS_PER_SM)
    nf4_dequant_batched_kernel(const DqParams* __restrict__ params,
                               const int64_t* __restrict__ iter_start, int32_t n_jobs) {
  __shared__ __align__(128) uint8_t stage[DQ2_WARPS][4096];
  const int warp = threadIdx.x >> 5;
  const int64_t total = __ldg(iter_start + n_jobs);
  int job = -1;
  int64_t job_lo = 0, job_hi = 0, nchunks = 0;
  DqParams p;
  float code[16];
  for (int64_t it = int64_t(blockIdx.x) * DQ2_WARPS + warp; it < total;
       it += int64_t(gridDim.x) * DQ2_WARPS) {
    if (it >= job_hi) {  // warp-uniform: advance to the job holding iteration `it`
      do {
        ++job;
        job_lo = __ldg(iter_start + job);
        job_hi = __ldg(iter_start + job + 1);
      } while (it >= job_hi && job + 1 < n_jobs);
      p = params[job];
      nchunks = p.nwords >> 3;
      load_code16(p.code, code);
    }
    dequant_iter_v2(p, nchunks, it - job_lo, code, stage[warp]);
  }
}

static int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = v > 0 ? v : 148;
  }
  return cached[dev];
}

// Chunk-kernel eligibility: fp16 out, whole 64-value chunks, 16-byte aligned buffers.
static bool chunk_path_ok(const DqParams& p) {
  return !p.f32out && (p.nwords % 8) == 0 && aligned(p.packed, 16) && aligned(p.out, 16) &&
         aligned(p.code, 16);
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

bool pdl_enabled(cudaStream_t s) {
  const char* v = std::getenv("STEW_PDL");
  if (v != nullptr && v[0] == '0') return false;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cs) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return cs == cudaStreamCaptureStatusNone;
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (chunk_path_ok(p)) {
    const int64_t iters = (p.nwords / 8 + DQ2_CHUNKS_PER_ITER - 1) / DQ2_CHUNKS_PER_ITER;
    const int64_t want = (iters + DQ2_WARPS - 1) / DQ2_WARPS;
    const int64_t cap = int64_t(sm_count()) * DQ2_CTAS_PER_SM;
    nf4_dequant_chunk_kernel<<<unsigned(want < cap ? want : cap), DQ2_THREADS, 0, s>>>(p);
    return launch_status("nf4_dequant_chunk_kernel launch");
  }
  const int64_t ctas = (p.nwords + DQ_WORDS_PER_CTA - 1) / DQ_WORDS_PER_CTA;
  NF4B_RETURN_IF(ctas > 0x7FFFFFFFll, NF4B_ERR_UNSUPPORTED);
  const bool al = aligned(packed, 4) && aligned(out, 16);
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
    // the batched kernel has only the chunk path: fp16 out, 64-value chunks, aligned buffers
    NF4B_RETURN_IF(params[i].f32out || params[i].nwords % 8 != 0, NF4B_ERR_UNSUPPORTED);
    NF4B_RETURN_IF(!chunk_path_ok(params[i]), NF4B_ERR_ALIGNMENT);
    starts[i] = total;
    total += (params[i].nwords / 8 + DQ2_CHUNKS_PER_ITER - 1) / DQ2_CHUNKS_PER_ITER;
  }
  starts[n_jobs] = total;
  const int64_t want = (total + DQ2_WARPS - 1) / DQ2_WARPS;
  const int64_t cap = int64_t(sm_count()) * DQ2_CTAS_PER_SM;
  *n_ctas = want < cap ? want : cap;
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
  nf4_dequant_batched_kernel<<<unsigned(n_ctas), DQ2_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      params, starts, n_jobs);
  return launch_status("nf4_dequant_batched_kernel launch");
}
