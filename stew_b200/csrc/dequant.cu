// Standalone NF4 unpack (sm_100a).
//
// Same arithmetic as the reference's `_nf4_unpack` (evilandangry/stew,
// solution/nf4.py:30-50):
//   nested: scale = code2[absmax8[blk]] * absmax2[blk / bs2] + offset  (nf4.py:36-39)
//   plain : scale = absmax[blk]                                        (nf4.py:41)
//   out[2j] = code[b >> 4] * scale, out[2j+1] = code[b & 15] * scale    (nf4.py:45-47)
// fp32 math with one rounding per operation (explicit __fmul_rn / __fadd_rn, so
// no FMA contraction can change a bit), one rounding to the output dtype.
// nf4b_qstate.nested == 2 selects the contracted form of the nested scale instead,
// fmaf(code2[absmax8[blk]], absmax2[blk / bs2], offset) rounded once: what a GPU compiler may
// emit for nf4.py:36-39, and what the reference's own test tolerates with a mismatch
// fraction below 1e-4 (solution/test_nf4_unpack.py:29-30) -- a debug form for diffing
// against such a build.
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
// The main fp16 path is the bulk-async kernel further down (nf4_dequant_tma_kernel), for one
// tensor or, from a device-side plan, for many tensors in one launch.
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
  int32_t nested;   // 0 plain, 1 nested (multiply, then add), 2 nested (one fused multiply-add)
  int32_t f32out;
};

__device__ __forceinline__ float nested_scale(int32_t mode, float c2, float a2, float off) {
  return mode == 2 ? __fmaf_rn(c2, a2, off) : __fadd_rn(__fmul_rn(c2, a2), off);
}

static_assert(sizeof(nf4b_dequant_job) % 8 == 0, "job struct layout");

__device__ __forceinline__ float block_scale(const DqParams& p, int64_t blk) {
  if (p.nested) {
    const uint32_t q = __ldg(p.absmax8 + blk);
    const float c2 = __ldg(p.code2 + q);
    const float a2 = __ldg(p.absmax2 + (blk >> p.log2_bs2));
    return nested_scale(p.nested, c2, a2, __ldg(p.offset));
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

// ---------------------------------------------------------------- main path
// Work unit of the main path: 32 chunks of 64 values (one per lane of a warp), i.e. 1 KB of
// packed bytes and 4 KB of fp16 output.
constexpr int DQ_CHUNKS_PER_ITER = 32;

__device__ __forceinline__ void load_code16(const float* code, float (&c)[16]) {
  const float4* c4 = reinterpret_cast<const float4*>(code);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 v = __ldg(c4 + i);
    c[4 * i] = v.x; c[4 * i + 1] = v.y; c[4 * i + 2] = v.z; c[4 * i + 3] = v.w;
  }
}

// ------------------------------------------------------------ bulk-async kernel
// Main path for blocksizes >= 64 (one scale per 64-value chunk), fp16 out, aligned buffers.
// Each warp runs its own pipeline over a contiguous range of 32-chunk iterations (1 KB packed
// in, 4 KB fp16 out each):
//   * lane 0 streams the packed bytes of the next DQ3_IN iterations into a ring of 1 KB
//     shared-memory slots with cp.async.bulk (completion counted on one mbarrier per slot), so
//     the next iteration's reads are in flight while the warp decodes;
//   * the block scales (absmax8 -> code2 * absmax2 + offset, or the fp32 absmax) of the next
//     iteration are loaded into registers one iteration ahead, which takes the dependent
//     absmax8 -> code2 load chain off the critical path;
//   * each lane decodes its 64-value chunk into a linear 4 KB output stage -- at step j it
//     handles word j ^ (lane & 7), read straight from the shared slot, so the 16-byte stores of
//     the 8 lanes of a shared-memory wavefront hit 8 different bank groups -- and lane 0 writes
//     the stage back with one cp.async.bulk store; two stages alternate, a stage being reused
//     only after its previous store has been read out (cp.async.bulk.wait_group.read).
// Warps take runs of 8 consecutive iterations in turn (blocked-cyclic), which keeps the grid
// inside one window of the sweep and keeps job changes (a new table, new pointers) rare.
// All loads and stores carry an L2 evict-first policy (streaming data, touched once).
// Every mbarrier wait is bounded; on expiry the warp records g_dequant_error, waits (bounded)
// for the loads it has in flight and returns.
constexpr int DQ3_WARPS = 4;
constexpr int DQ3_THREADS = 32 * DQ3_WARPS;
// Pipeline depth and residency, measured on the whole-model sweep (B200): more resident warps
// beat deeper per-warp pipelines -- 2 packed slots x 5 CTAs (20 warps) 5,756 GB/s, 3 x 5
// 5,674, 4 x 4 5,634, 5 x 4 5,583; single output stages with 6-7 CTAs (registers spill)
// 5,381-5,478.
constexpr int DQ3_IN = 2;    // packed slots per warp, 1 KB each
constexpr int DQ3_OUT = 2;   // output stages per warp, 4 KB each
constexpr int DQ3_WARP_BYTES = DQ3_OUT * 4096 + DQ3_IN * 1024;
constexpr int DQ3_RING = 8;  // tickets a warp's producer may hold ahead (dynamic walk)
constexpr int DQ3_SMEM = DQ3_WARPS * DQ3_WARP_BYTES + DQ3_WARPS * DQ3_IN * 8 + DQ3_WARPS * DQ3_RING * 4;
// Resident CTAs per SM: 5 (20 warps; 5 x 41 KB of shared memory, <= 102 registers a thread)
// for blocksizes >= 64, 4 for plans with blocksize 32 (two tables per chunk need more
// registers).
template <bool TWO>
constexpr int dq3_ctas_per_sm() { return TWO ? 4 : 5; }
// Run length of the blocked-cyclic walk: iterations (4 KB of output each) a warp takes in a
// row.  Measured: 1 -> 4,802 GB/s, 2 -> 5,213, 4 -> 5,470, 8 -> 5,564, 16 -> 5,573, 64 -> 5,317,
// one contiguous range per warp -> 5,404 (3 packed slots, no L2 hint); 8 with the hint: 5,636.
constexpr int DQ3_RUN = 8;
constexpr long long DQ3_WAIT_CYCLES = 4000000000ll;  // ~2 s

__device__ int g_dequant_error;

// Streaming data is read and written once: both directions carry an L2 evict-first policy
// (+1.3 % on the whole-model sweep).
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void bulk_load_1d(uint32_t smem_dst, const void* src, uint32_t bytes,
                                             uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void bulk_store_1d(void* dst, uint32_t smem_src, uint32_t bytes, uint64_t pol) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group.L2::cache_hint [%0], [%1], %2, %3;" ::"l"(dst),
               "r"(smem_src), "r"(bytes), "l"(pol)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// All but the last N bulk stores have finished reading their shared-memory stages.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ bool dq3_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait_sleep(bar, parity, 20000u)) {
    if (clock64() - t0 > DQ3_WAIT_CYCLES) {
      atomicExch(&g_dequant_error, 1);
      return false;
    }
  }
  return true;
}

// Job cursor over the prefix sums of iterations (n_jobs == 0: the single job of the launch).
struct Dq3Jobs {
  const DqParams* params;
  const int64_t* start;
  int32_t n;
  __device__ __forceinline__ int64_t lo(int j) const { return start ? __ldg(start + j) : 0; }
  __device__ __forceinline__ int64_t hi(int j) const {
    return start ? __ldg(start + j + 1) : ((params->nwords >> 3) + DQ_CHUNKS_PER_ITER - 1) / DQ_CHUNKS_PER_ITER;
  }
  // The job holding iteration `it`: the last job whose first iteration is <= it, found by the
  // whole warp (32 probes per round, so two dependent loads for up to 1,024 jobs).  Call from
  // all 32 lanes with the same `it`.
  __device__ __forceinline__ int find(int64_t it) const {
    const int lane = threadIdx.x & 31;
    int a = 0, b = n - 1;  // the answer lies in [a, b]
    while (a < b) {
      const int step = (b - a + 32) / 32;  // ceil((b - a + 1) / 32)
      const int m = min(a + lane * step, b);
      const uint32_t le = __ballot_sync(0xffffffffu, lo(m) <= it);
      const int last = 31 - __clz(le);  // lane 0 always qualifies (lo(a) <= it)
      a = min(a + last * step, b);
      b = min(b, a + step - 1);
    }
    return a;
  }
};

// Scale sources of one 64-value chunk: its block (blocksize >= 64), or its two 32-value
// blocks (blocksize 32; the second pair is the first one otherwise).
struct Dq3Src {
  uint32_t q0, q1;
  float a0, a1;
};

// TWO: the launch has blocksize-32 jobs, whose chunks span two blocks; for the other jobs of
// such a launch the second block is the first one again.
template <bool TWO>
__device__ __forceinline__ Dq3Src dq3_scale_src(const DqParams& p, int64_t chunk, bool valid) {
  Dq3Src r{0u, 0u, 0.f, 0.f};
  if (!valid) return r;
  const int64_t blk = (chunk << 6) >> p.log2_bs;
  if (p.nested) {
    r.q0 = __ldg(p.absmax8 + blk);
    r.a0 = __ldg(p.absmax2 + (blk >> p.log2_bs2));
  } else {
    r.a0 = __ldg(p.absmax32 + blk);
  }
  if (TWO) {
    const int64_t blk1 = p.log2_bs == 5 ? blk + 1 : blk;
    if (p.nested) {
      r.q1 = __ldg(p.absmax8 + blk1);
      r.a1 = __ldg(p.absmax2 + (blk1 >> p.log2_bs2));
    } else {
      r.a1 = __ldg(p.absmax32 + blk1);
    }
  }
  return r;
}

__device__ __forceinline__ float dq3_scale(const DqParams& p, uint32_t q, float a, float off) {
  return p.nested ? nested_scale(p.nested, __ldg(p.code2 + q), a, off) : a;
}

// TWO: blocksize 32 (two blocks, two tables per chunk); otherwise every job of the launch has
// blocksize >= 64.
template <bool TWO>
__global__ void __launch_bounds__(DQ3_THREADS, dq3_ctas_per_sm<TWO>())
    nf4_dequant_tma_kernel(const DqParams* __restrict__ params, const int64_t* __restrict__ iter_start,
                           int32_t n_jobs, uint32_t* __restrict__ work,
                           const __grid_constant__ DqParams single) {
  extern __shared__ __align__(128) uint8_t dq3_smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t out_s = smem_u32(dq3_smem + warp * DQ3_WARP_BYTES);
  const uint32_t in_s = out_s + DQ3_OUT * 4096;
  uint64_t* bars = reinterpret_cast<uint64_t*>(dq3_smem + DQ3_WARPS * DQ3_WARP_BYTES) + warp * DQ3_IN;
  volatile int32_t* ring = reinterpret_cast<volatile int32_t*>(
                               dq3_smem + DQ3_WARPS * DQ3_WARP_BYTES + DQ3_WARPS * DQ3_IN * 8) +
                           warp * DQ3_RING;
  const Dq3Jobs J{n_jobs > 0 ? params : &single, n_jobs > 0 ? iter_start : nullptr, n_jobs > 0 ? n_jobs : 1};
  const int64_t total = J.start ? J.lo(J.n) : J.hi(0);
  const int64_t nw = int64_t(gridDim.x) * DQ3_WARPS;
  const int64_t wid = int64_t(blockIdx.x) * DQ3_WARPS + warp;
  constexpr int64_t bl = DQ3_RUN;
  const uint64_t pol = l2_evict_first();
  // Static walk (a launch without a work counter): blocked-cyclic rounds in which every warp
  // takes a run of DQ3_RUN consecutive iterations, so at any time the grid works inside one
  // window of the sweep (DRAM pages are shared) and a warp's iterations still come in runs (few
  // job changes, scale prefetch); what is left after the whole rounds is dealt in one last
  // round of shorter runs (ceil(rest / warps) each).  -1 ends a warp's walk.
  const int64_t rounds = total / (nw * bl);
  const int64_t tail0 = rounds * nw * bl;            // first iteration of the last round
  const int64_t bl2 = (total - tail0 + nw - 1) / nw;  // run length of the last round
  const int64_t t0 = tail0 + wid * bl2;               // this warp's run in the last round
  const int64_t t1 = min64(t0 + bl2, total);
  auto next_static = [&](int64_t it) -> int64_t {
    if (it >= tail0) return it + 1 < t1 ? it + 1 : -1;
    if ((it + 1) % bl) return it + 1;
    const int64_t nx = it + 1 + (nw - 1) * bl;
    return nx < tail0 ? nx : (t0 < t1 ? t0 : -1);
  };
  // Dynamic walk (a batched plan's work counter): a warp takes the next ticket when it needs
  // one -- runs of DQ3_RUN iterations in sweep order, then single iterations for the last
  // ~2 per warp -- so warps that the SM's scheduler favours take more of the work instead of
  // finishing early and leaving the last CTAs of every SM to run alone.  Lane 0 (the producer,
  // which runs DQ3_IN iterations ahead) takes the tickets and keeps them in a per-warp ring in
  // shared memory, where the consumer lanes read them after a __syncwarp.
  const int64_t tail_n = min64(total, 2 * nw);
  const int64_t n_runs = (total - tail_n) / bl;
  const int64_t dyn0 = n_runs * bl;                   // first single-iteration ticket
  const int64_t n_tickets = n_runs + (total - dyn0);
  auto t_lo = [&](int32_t t) -> int64_t { return t < n_runs ? int64_t(t) * bl : dyn0 + (t - n_runs); };
  auto t_hi = [&](int32_t t) -> int64_t { return t < n_runs ? int64_t(t) * bl + bl : dyn0 + (t - n_runs) + 1; };
  auto grab = [&]() -> int32_t {  // lane 0
    const uint32_t t = atomicAdd(work, 1u);
    return int64_t(t) < n_tickets ? int32_t(t) : -1;
  };

  if (lane == 0) {
    for (int i = 0; i < DQ3_IN; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
    if (work != nullptr) ring[0] = grab();
  }
  __syncwarp();
  // the warp's first iteration (-1: none) -- both cursors start there
  int64_t first;
  if (work != nullptr) {
    const int32_t t = ring[0];
    first = t >= 0 ? t_lo(t) : -1;
  } else {
    first = rounds > 0 ? wid * bl : (t0 < t1 ? t0 : -1);
  }

  // producer cursor (lane 0): the next iteration to load (-1: none), its ticket's end and ring
  // position, and its job
  int64_t pit = first, pend = (work != nullptr && first >= 0) ? t_hi(ring[0]) : 0;
  uint32_t pr = 0;
  int pj = first >= 0 ? J.find(first) : 0;
  int64_t plo = J.lo(pj), phi = J.hi(pj);
  int64_t issued = 0;
  auto issue = [&]() {  // lane 0: loads iteration pit into slot issued % DQ3_IN, then advances
    while (pit >= phi) {
      ++pj;
      plo = phi;
      phi = J.hi(pj);
    }
    const uint8_t* packed = J.params[pj].packed;
    const int64_t nch = J.params[pj].nwords >> 3;
    const int64_t li = pit - plo;
    const uint32_t bytes = uint32_t(min64(DQ_CHUNKS_PER_ITER, nch - li * DQ_CHUNKS_PER_ITER)) * 32u;
    const int s = int(issued % DQ3_IN);
    mbar_arrive_expect_tx(&bars[s], bytes);
    bulk_load_1d(in_s + uint32_t(s) * 1024u, packed + li * 1024, bytes, smem_u32(&bars[s]), pol);
    ++issued;
    if (work == nullptr) {
      pit = next_static(pit);
    } else if (++pit == pend) {
      const int32_t t = grab();
      ring[++pr & (DQ3_RING - 1)] = t;
      pit = t >= 0 ? t_lo(t) : -1;
      pend = t >= 0 ? t_hi(t) : 0;
    }
  };
  if (lane == 0)
    while (issued < DQ3_IN && pit >= 0) issue();
  __syncwarp();
  // run-time 1 << 16 and 1 << 31 for the decode's multiply-high shifts (nf4_decode.cuh)
  const uint32_t k16 = 1u << (16 + (n_jobs < 0));
  const uint32_t k31 = k16 << 15;

  // consumer cursor (all lanes, warp-uniform): the iteration, its ticket's end and ring position
  int64_t it = first;
  int64_t cend = pend;
  uint32_t cr = 0;
  if (work != nullptr && first >= 0) cend = t_hi(ring[0]);
  auto peek = [&](int64_t i) -> int64_t {  // the iteration after i in this warp's walk
    if (work == nullptr) return next_static(i);
    if (i + 1 < cend) return i + 1;
    const int32_t t = ring[(cr + 1) & (DQ3_RING - 1)];
    return t >= 0 ? t_lo(t) : -1;
  };
  int cj = -1;
  int64_t clo = 0, chi = 0;
  DqParams p;
  float code[16];
  float off = 0.f;
  Dq3Src pre{0u, 0u, 0.f, 0.f};
  bool have_pre = false;
  int64_t k = 0;
  bool ok = true;
  int s = 0;          // slot of iteration k (k % DQ3_IN) and the phase of its barrier
  uint32_t ph = 0;
  for (; it >= 0; ++k) {
    if (it >= chi) {
      cj = (cj < 0) ? J.find(it) : cj + 1;
      while (J.hi(cj) <= it) ++cj;
      clo = J.lo(cj);
      chi = J.hi(cj);
      p = J.params[cj];
      load_code16(p.code, code);
      off = p.nested ? __ldg(p.offset) : 0.f;
      have_pre = false;
    }
    const int64_t li = it - clo;
    const int64_t nch = p.nwords >> 3;
    const int nvalid = int(min64(DQ_CHUNKS_PER_ITER, nch - li * DQ_CHUNKS_PER_ITER));
    const int64_t ch = li * DQ_CHUNKS_PER_ITER + lane;
    const bool valid = lane < nvalid;
    const Dq3Src cur = have_pre ? pre : dq3_scale_src<TWO>(p, ch, valid);
    // the next iteration's scale sources, while it belongs to the same job
    const int64_t it1 = peek(it);
    have_pre = it1 >= 0 && it1 < chi;
    if (have_pre) {
      const int64_t li1 = it1 - clo;
      const int nv1 = int(min64(DQ_CHUNKS_PER_ITER, nch - li1 * DQ_CHUNKS_PER_ITER));
      pre = dq3_scale_src<TWO>(p, li1 * DQ_CHUNKS_PER_ITER + lane, lane < nv1);
    }
    const float sc0 = valid ? dq3_scale(p, cur.q0, cur.a0, off) : 0.f;
    const Nf4Table t0 = make_table(code, sc0);
    const Nf4Table t1 = TWO ? make_table(code, valid ? dq3_scale(p, cur.q1, cur.a1, off) : 0.f) : t0;

    ok = __all_sync(0xffffffffu, dq3_wait(&bars[s], ph));
    if (!ok) break;
    // the output stage written DQ3_OUT iterations ago has been read out by its store
    if (lane == 0 && k >= DQ3_OUT) bulk_wait_read<DQ3_OUT - 1>();
    __syncwarp();
    const uint32_t stage = out_s + uint32_t(k % DQ3_OUT) * 4096u;
    const uint32_t src = in_s + uint32_t(s) * 1024u + uint32_t(lane) * 32u;
    const uint32_t dst = stage + uint32_t(lane) * 128u;
    const uint32_t key = uint32_t(lane & 7);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t jj = uint32_t(j) ^ key;
      uint32_t w;
      asm volatile("ld.shared.b32 %0, [%1];" : "=r"(w) : "r"(src + jj * 4u));
      uint4 v;
      if (!TWO) {
        v = decode_word_f16_mh(t0, w, k16, k31);
      } else {
        // blocksize 32: words 0-3 of the chunk are the first block, 4-7 the second
        const bool hi = jj >= 4u;
        Nf4Table t;
        t.l0 = hi ? t1.l0 : t0.l0; t.l1 = hi ? t1.l1 : t0.l1; t.l2 = hi ? t1.l2 : t0.l2;
        t.l3 = hi ? t1.l3 : t0.l3; t.h0 = hi ? t1.h0 : t0.h0; t.h1 = hi ? t1.h1 : t0.h1;
        t.h2 = hi ? t1.h2 : t0.h2; t.h3 = hi ? t1.h3 : t0.h3;
        v = decode_word_f16_mh(t, w, k16, k31);
      }
      asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(dst + jj * 16u), "r"(v.x), "r"(v.y),
                   "r"(v.z), "r"(v.w)
                   : "memory");
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      bulk_store_1d(static_cast<uint8_t*>(p.out) + li * 4096, stage, uint32_t(nvalid) * 128u, pol);
      // slot s has been read by every lane: refill it with the walk's next unloaded iteration
      if (pit >= 0) issue();
    }
    if (++s == DQ3_IN) {
      s = 0;
      ph ^= 1u;
    }
    // advance the consumer cursor (a new ticket's ring entry was written when the producer
    // loaded the iteration before it, at least one __syncwarp ago)
    if (work == nullptr) {
      it = next_static(it);
    } else if (++it == cend) {
      const int32_t t = ring[++cr & (DQ3_RING - 1)];
      it = t >= 0 ? t_lo(t) : -1;
      cend = t >= 0 ? t_hi(t) : 0;
    }
  }
  if (!ok && lane == 0) {
    // loads still in flight land in this warp's slots: wait for them (bounded) before leaving
    for (int64_t j = k; j < issued; ++j) {
      if (!dq3_wait(&bars[s], ph)) break;
      if (++s == DQ3_IN) {
        s = 0;
        ph ^= 1u;
      }
    }
  }
  if (lane == 0) bulk_wait_all();
  __syncwarp();
  if (work != nullptr && lane == 0) {
    // the last warp of the launch leaves the plan's work counter at zero for its next launch
    __threadfence();
    if (atomicAdd(work + 1, 1u) == uint32_t(nw) - 1u) {
      work[0] = 0u;
      work[1] = 0u;
      __threadfence();
    }
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

// Main-path eligibility: fp16 out, whole 64-value chunks, 16-byte aligned buffers (the bulk
// copies move whole 16-byte units between 16-byte aligned addresses).
static bool chunk_path_ok(const DqParams& p) {
  return !p.f32out && (p.nwords % 8) == 0 && aligned(p.packed, 16) && aligned(p.out, 16) &&
         aligned(p.code, 16);
}

// Launch descriptor bit of nf4b_dequant_plan / nf4b_dequant_batched: the plan has a job of
// blocksize 32 and runs the two-table variant.
constexpr int64_t kDq3TwoFlag = int64_t(1) << 32;

static int64_t dq3_iters(const DqParams& p) {
  return ((p.nwords >> 3) + DQ_CHUNKS_PER_ITER - 1) / DQ_CHUNKS_PER_ITER;
}

// CTAs of a main-path launch over `iters` iterations: enough for one iteration per warp, at
// most the resident CTAs of the variant on every SM.
static int64_t dq3_grid(int64_t iters, bool two) {
  const int64_t want = (iters + DQ3_WARPS - 1) / DQ3_WARPS;
  const int64_t cap = int64_t(sm_count()) * (two ? dq3_ctas_per_sm<true>() : dq3_ctas_per_sm<false>());
  return want < cap ? want : cap;
}

// The main path's dynamic shared memory (above the 48 KB default) on the current device.
static int dq3_smem_attr() {
  static std::mutex mu;
  static bool done[64] = {false};
  int dev = 0;
  NF4B_CUDA_TRY(cudaGetDevice(&dev));
  NF4B_RETURN_IF(dev < 0 || dev >= 64, NF4B_ERR_DEVICE);
  std::lock_guard<std::mutex> lock(mu);
  if (!done[dev]) {
    NF4B_CUDA_TRY(cudaFuncSetAttribute(nf4_dequant_tma_kernel<false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, DQ3_SMEM));
    NF4B_CUDA_TRY(cudaFuncSetAttribute(nf4_dequant_tma_kernel<true>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, DQ3_SMEM));
    done[dev] = true;
  }
  return NF4B_OK;
}

// ------------------------------------------------------------------- host side
static int check_qstate(const nf4b_qstate* qs, int32_t* log2_bs, int32_t* log2_bs2) {
  NF4B_RETURN_IF(qs == nullptr || qs->code == nullptr, NF4B_ERR_INVALID_ARG);
  const int lb = ilog2_exact(qs->blocksize);
  NF4B_RETURN_IF(lb < 5 || lb > 8, NF4B_ERR_UNSUPPORTED);  // 32, 64, 128, 256 (nf4.py:66)
  *log2_bs = lb;
  *log2_bs2 = 0;
  NF4B_RETURN_IF(qs->nested < 0 || qs->nested > 2, NF4B_ERR_INVALID_ARG);
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
  NF4B_RETURN_IF(out_dtype != NF4B_F16 && out_dtype != NF4B_F32, NF4B_ERR_UNSUPPORTED);
  NF4B_RETURN_IF(numel < 0, NF4B_ERR_INVALID_ARG);
  if (numel == 0) {  // an empty tensor: nothing is read or written, its pointers may be NULL
    NF4B_RETURN_IF(qs == nullptr, NF4B_ERR_INVALID_ARG);
    const int lb = ilog2_exact(qs->blocksize);
    NF4B_RETURN_IF(lb < 5 || lb > 8, NF4B_ERR_UNSUPPORTED);
    *p = DqParams{packed, out, nullptr, nullptr, nullptr, nullptr, nullptr, qs->code, 0, lb, 8,
                  qs->nested, out_dtype == NF4B_F32};
    return NF4B_OK;
  }
  NF4B_RETURN_IF(packed == nullptr || out == nullptr, NF4B_ERR_INVALID_ARG);
  int32_t lb = 0, lb2 = 0;
  int st = check_qstate(qs, &lb, &lb2);
  if (st != NF4B_OK) return st;
  NF4B_RETURN_IF(numel % qs->blocksize != 0, NF4B_ERR_UNSUPPORTED);  // nf4.py:69
  *p = DqParams{packed, out, qs->absmax8, qs->absmax32, qs->code2, qs->absmax2, qs->offset,
                qs->code, numel >> 3, lb, lb2, qs->nested, out_dtype == NF4B_F32};
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
    st = dq3_smem_attr();
    if (st != NF4B_OK) return st;
    const bool two = p.log2_bs == 5;
    const unsigned grid = unsigned(dq3_grid(dq3_iters(p), two));
    if (two)
      nf4_dequant_tma_kernel<true><<<grid, DQ3_THREADS, DQ3_SMEM, s>>>(nullptr, nullptr, 0, nullptr, p);
    else
      nf4_dequant_tma_kernel<false><<<grid, DQ3_THREADS, DQ3_SMEM, s>>>(nullptr, nullptr, 0, nullptr, p);
    return launch_status("nf4_dequant_tma_kernel launch");
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

// Plan layout: the jobs' parameters, the prefix sums of their iterations (n_jobs + 1), then
// the launch's work counter (next ticket, finished warps; zero between launches).
static int64_t plan_work_offset(int32_t n_jobs) {
  return int64_t(n_jobs) * int64_t(sizeof(DqParams)) + int64_t(n_jobs + 1) * 8;
}

extern "C" int64_t nf4b_dequant_plan_bytes(int32_t n_jobs) {
  if (n_jobs <= 0) return 0;
  return plan_work_offset(n_jobs) + 16;
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
    total += dq3_iters(params[i]);
  }
  starts[n_jobs] = total;
  NF4B_RETURN_IF(total > 0x7FFFFFFFll, NF4B_ERR_UNSUPPORTED);  // tickets are 32-bit
  // the launch descriptor: CTA count, and bit 32 for the blocksize-32 variant
  bool two = false;
  for (int i = 0; i < n_jobs; ++i) two = two || (params[i].nwords > 0 && params[i].log2_bs == 5);
  *n_ctas = dq3_grid(total, two) | (two ? kDq3TwoFlag : 0);
  // A copy from pageable host memory returns once the source has been staged,
  // so the local buffer may be released right after.
  NF4B_CUDA_TRY(cudaMemcpyAsync(plan_dev, host.data(), host.size(), cudaMemcpyHostToDevice,
                                static_cast<cudaStream_t>(stream)));
  return NF4B_OK;
}

extern "C" int nf4b_dequant_batched(const void* plan_dev, int32_t n_jobs, int64_t launch,
                                    void* stream) {
  NF4B_RETURN_IF(plan_dev == nullptr || n_jobs <= 0 || launch < 0, NF4B_ERR_INVALID_ARG);
  const bool two = (launch & kDq3TwoFlag) != 0;
  const int64_t n_ctas = launch & ~kDq3TwoFlag;
  NF4B_RETURN_IF(n_ctas > 0x7FFFFFFFll, NF4B_ERR_UNSUPPORTED);
  if (n_ctas == 0) return NF4B_OK;
  int st = check_device();
  if (st != NF4B_OK) return st;
  const DqParams* params = static_cast<const DqParams*>(plan_dev);
  const int64_t* starts = reinterpret_cast<const int64_t*>(
      static_cast<const uint8_t*>(plan_dev) + size_t(n_jobs) * sizeof(DqParams));
  st = dq3_smem_attr();
  if (st != NF4B_OK) return st;
  uint32_t* work = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(const_cast<void*>(plan_dev)) +
                                               plan_work_offset(n_jobs));
  DqParams none{};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (two)
    nf4_dequant_tma_kernel<true><<<unsigned(n_ctas), DQ3_THREADS, DQ3_SMEM, s>>>(params, starts, n_jobs, work, none);
  else
    nf4_dequant_tma_kernel<false><<<unsigned(n_ctas), DQ3_THREADS, DQ3_SMEM, s>>>(params, starts, n_jobs, work, none);
  return launch_status("nf4_dequant_tma_kernel launch");
}

extern "C" int nf4b_dequant_error_flag(int* value, int reset) {
  NF4B_RETURN_IF(value == nullptr, NF4B_ERR_INVALID_ARG);
  NF4B_CUDA_TRY(cudaMemcpyFromSymbol(value, g_dequant_error, sizeof(int)));
  if (reset) {
    const int zero = 0;
    NF4B_CUDA_TRY(cudaMemcpyToSymbol(g_dequant_error, &zero, sizeof(int)));
  }
  return NF4B_OK;
}
