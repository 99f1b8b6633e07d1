// LoRA (rank 16) side kernels of the q/v adapter (peft lora.Linear,
// y = base(x) + lora_B(lora_A(x)) * scaling; the reference keeps peft's module and
// only touches its input cast, solution/rmsnorm.py:137-150).
//
//  lora_project16   out[t, r] = sum_k act[t, k] * W[r, k]       (X A^T forward, dY B backward)
//                   fp32 accumulate, fp16 result (what peft's fp16 autocast linear yields).
//                   HBM-bound on `act`; mma.sync tiles of 16 tokens, K split over 8 warps.
//  lora_grads16     G[r, c] = sum_t P[t, r] * Q[t, c]            (the two weight gradients)
//                   split over columns and tokens; the token ranges' fp32 partials go to
//                   caller-provided scratch and the last CTA of each column tile adds them up
//                   in a fixed order and applies the scale (one launch, deterministic).
#include <mutex>

#include "common.cuh"
#include "stew_nf4.h"

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

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// W(r, k .. k+7) as 8 halves (k a multiple of 8) of a K-contiguous weight (forward: lora A
// [16, in]): one 16-byte load.
__device__ __forceinline__ uint4 ld_w8(const __half* w, int64_t sr, int r, int64_t k) {
  return __ldg(reinterpret_cast<const uint4*>(w + r * sr + k));
}

// Strided weight (backward: lora B [out, 16], K = out, one 32-byte row per k): a warp stages the
// rows of up to LP_STAGE_CHUNKS chunks of its K slice in shared memory with cp.async (the two
// 16-byte halves of row k swapped when bit 3 of k is set, so the eight rows an ldmatrix reads
// fall in four bank groups) and reads each chunk's fragments with two ldmatrix .trans.
constexpr int LP_STAGE_CHUNKS = 8;
constexpr int LP_STAGE_BYTES = LP_STAGE_CHUNKS * 32 * 32;  // per warp

// Thread (g, c) of a warp reads, per 32-wide K chunk j, the 8 consecutive values
// [32 j + 8 c, +8) of token rows g and g+8 (two 16-byte loads) and feeds them to two k16 MMA
// steps: fragment position 2c(+1) takes values 0-1 (step 0) / 4-5 (step 1), position
// 2c+8(+9) values 2-3 / 6-7.  The adapter weight is read with the same assignment, so both
// operands see one permutation of K and the dot products are those of the natural order.
// WK: the weight is K-contiguous (sk == 1); otherwise it is [kdim][16] (sr == 1, sk == 16).
// One projection of a launch (blockIdx.y picks it; all of a launch's share n and WK).
struct ProjJob {
  const __half* act;
  const __half* w;
  int64_t sr, sk;
  __half* out;
  int64_t kdim;
};
constexpr int LP_MAX_JOBS = 3;
struct ProjJobs {
  ProjJob j[LP_MAX_JOBS];
};

template <bool WK>
__global__ void __launch_bounds__(LP_THREADS)
    lora_project16_kernel(const __grid_constant__ ProjJobs jobs, int64_t n) {
  grid_dep_wait();  // programmatic launch: no global access before the wait
  const ProjJob& job = jobs.j[blockIdx.y];
  const __half* __restrict__ act = job.act;
  const __half* __restrict__ w = job.w;
  const int64_t sr = job.sr, kdim = job.kdim;  // sk is 1 (WK) or 16, fixed by the layout
  __half* __restrict__ out = job.out;
  __shared__ float red[LP_WARPS][LP_TOK][17];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;  // mma fragment coordinates
  const int64_t t0 = int64_t(blockIdx.x) * LP_TOK;
  const int64_t chunks = kdim / 32;
  const int64_t per = (chunks + LP_WARPS - 1) / LP_WARPS;
  const int64_t jb = warp * per;
  const int64_t je = min64(chunks, jb + per);
  const bool v0 = t0 + g < n, v1 = t0 + g + 8 < n;
  const uint4* x0 = reinterpret_cast<const uint4*>(act + (t0 + g) * kdim);
  const uint4* x1 = reinterpret_cast<const uint4*>(act + (t0 + g + 8) * kdim);
  float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
  auto mma_chunk = [&](const uint4& xa, const uint4& xb, uint32_t w0x, uint32_t w0y, uint32_t w0z,
                       uint32_t w0w, uint32_t w1x, uint32_t w1y, uint32_t w1z, uint32_t w1w) {
    const uint32_t s0[4] = {xa.x, xb.x, xa.y, xb.y};
    const uint32_t s1[4] = {xa.z, xb.z, xa.w, xb.w};
    mma16816(d0, s0, w0x, w0y);
    mma16816(d1, s0, w1x, w1y);
    mma16816(d0, s1, w0z, w0w);
    mma16816(d1, s1, w1z, w1w);
  };
  // chunks in batches of 4: every activation load of a batch is issued before its MMAs, so a
  // warp waits for memory about once per batch instead of once per chunk
  constexpr int LP_BATCH = 4;
  if (WK) {
    for (int64_t j0 = jb; j0 < je; j0 += LP_BATCH) {
      uint4 xa[LP_BATCH], xb[LP_BATCH], w0[LP_BATCH], w1[LP_BATCH];
#pragma unroll
      for (int u = 0; u < LP_BATCH; ++u) {
        const int64_t k = 32 * (j0 + u) + 8 * c;
        const bool in = j0 + u < je;
        xa[u] = (in && v0) ? __ldg(x0 + (k >> 3)) : make_uint4(0, 0, 0, 0);
        xb[u] = (in && v1) ? __ldg(x1 + (k >> 3)) : make_uint4(0, 0, 0, 0);
        w0[u] = in ? ld_w8(w, sr, g, k) : make_uint4(0, 0, 0, 0);      // adapter rows 0-7 (d0)
        w1[u] = in ? ld_w8(w, sr, 8 + g, k) : make_uint4(0, 0, 0, 0);  // adapter rows 8-15 (d1)
      }
#pragma unroll
      for (int u = 0; u < LP_BATCH; ++u)
        mma_chunk(xa[u], xb[u], w0[u].x, w0[u].y, w0[u].z, w0[u].w, w1[u].x, w1[u].y, w1[u].z, w1[u].w);
    }
  } else {
    // the launch holds LP_WARPS regions of min(per, LP_STAGE_CHUNKS) KB for the job with the
    // longest K; this job's per is at most that job's
    extern __shared__ __align__(128) uint8_t lp_stage[];
    const int64_t stage_chunks = per < LP_STAGE_CHUNKS ? per : LP_STAGE_CHUNKS;
    const uint32_t wb = smem_u32(lp_stage) + uint32_t(warp) * uint32_t(stage_chunks) * 1024u;
    // ldmatrix x4: lane l gives row l % 8 of matrix l / 8; matrix m holds, for fragment rows
    // 2c and 2c+1, the weight rows 8 c + 2 m and 8 c + 2 m + 1 of the chunk (values 2m, 2m+1 of
    // each lane's 8), i.e. row 8 (i / 2) + (i % 2) + 2 m for i = l % 8
    const int lrow = 8 * ((lane & 7) >> 1) + (lane & 1) + 2 * (lane >> 3);
    for (int64_t r0 = jb; r0 < je; r0 += stage_chunks) {
      const int64_t r1 = min64(je, r0 + stage_chunks);
      const int pieces = int(r1 - r0) * 64;  // 32 rows a chunk, two 16-byte halves a row
      __syncwarp();  // the previous round's ldmatrix reads are done
      for (int p = lane; p < pieces; p += 32) {
        const int row = p >> 1, half = p & 1;
        cp_async16(wb + uint32_t(row * 32 + ((half ^ ((row >> 3) & 1)) << 4)),
                   w + (32 * r0 + row) * 16 + 8 * half, true);
      }
      cp_async_commit();
      for (int64_t j0 = r0; j0 < r1; j0 += LP_BATCH) {
        uint4 xa[LP_BATCH], xb[LP_BATCH];
#pragma unroll
        for (int u = 0; u < LP_BATCH; ++u) {
          const int64_t k = 32 * (j0 + u) + 8 * c;
          const bool in = j0 + u < r1;
          xa[u] = (in && v0) ? __ldg(x0 + (k >> 3)) : make_uint4(0, 0, 0, 0);
          xb[u] = (in && v1) ? __ldg(x1 + (k >> 3)) : make_uint4(0, 0, 0, 0);
        }
        if (j0 == r0) {
          cp_async_wait<0>();
          __syncwarp();
        }
#pragma unroll
        for (int u = 0; u < LP_BATCH; ++u) {
          if (j0 + u >= r1) break;
          const int row = int(j0 + u - r0) * 32 + lrow;
          const uint32_t rb = wb + uint32_t(row * 32);
          const uint32_t sw = uint32_t((row >> 3) & 1) << 4;
          uint32_t b0[4], b1[4];
          ldsm_x4_t(rb + sw, b0);          // adapter rows (ranks) 0-7
          ldsm_x4_t(rb + (sw ^ 16u), b1);  // ranks 8-15
          mma_chunk(xa[u], xb[u], b0[0], b0[1], b0[2], b0[3], b1[0], b1[1], b1[2], b1[3]);
        }
      }
    }
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

// Several rank-16 projections over the same n tokens in one launch (the adapters of a grouped
// forward, X A_i^T, or of a grouped backward, dY_i B_i); every job's weight has the same
// layout (K-contiguous or not).
int lora_project16_multi(const void* const* act, const void* const* w, int64_t w_stride_r,
                         int64_t w_stride_k, void* const* out, const int64_t* kdim, int n_jobs,
                         int64_t n, cudaStream_t s) {
  NF4B_RETURN_IF(n_jobs < 1 || n_jobs > LP_MAX_JOBS, NF4B_ERR_UNSUPPORTED);
  // the two weight layouts the kernels take: K-contiguous [16][kdim] or [kdim][16]
  const bool wk = w_stride_k == 1;
  NF4B_RETURN_IF(!wk && (w_stride_r != 1 || w_stride_k != 16), NF4B_ERR_UNSUPPORTED);
  ProjJobs js{};
  int64_t kmax = 0;
  for (int i = 0; i < n_jobs; ++i) {
    NF4B_RETURN_IF(kdim[i] % 32 != 0, NF4B_ERR_UNSUPPORTED);
    NF4B_RETURN_IF(!aligned(act[i], 16) || !aligned(w[i], 16), NF4B_ERR_ALIGNMENT);
    js.j[i] = ProjJob{static_cast<const __half*>(act[i]), static_cast<const __half*>(w[i]), w_stride_r,
                      w_stride_k, static_cast<__half*>(out[i]), kdim[i]};
    kmax = kdim[i] > kmax ? kdim[i] : kmax;
  }
  if (n == 0) return NF4B_OK;
  const int64_t ctas = (n + LP_TOK - 1) / LP_TOK;
  NF4B_RETURN_IF(ctas > 0x7FFFFFFFll, NF4B_ERR_UNSUPPORTED);
  const dim3 grid{unsigned(ctas), unsigned(n_jobs), 1u};
  if (wk) {
    NF4B_CUDA_TRY(launch_pdl(lora_project16_kernel<true>, dim3(grid), dim3(LP_THREADS), size_t(0),
                             s, js, n));
  } else {
    // each warp stages up to LP_STAGE_CHUNKS chunks of its K slice at a time
    const int64_t per = (kmax / 32 + LP_WARPS - 1) / LP_WARPS;
    const size_t smem = size_t(LP_WARPS) * size_t(per < LP_STAGE_CHUNKS ? per : LP_STAGE_CHUNKS) * 1024;
    {
      static std::mutex mu;
      static bool done[64] = {false};
      int dev = 0;
      NF4B_CUDA_TRY(cudaGetDevice(&dev));
      NF4B_RETURN_IF(dev < 0 || dev >= 64, NF4B_ERR_DEVICE);
      std::lock_guard<std::mutex> lock(mu);
      if (!done[dev]) {
        NF4B_CUDA_TRY(cudaFuncSetAttribute(lora_project16_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           LP_WARPS * LP_STAGE_BYTES));
        done[dev] = true;
      }
    }
    NF4B_CUDA_TRY(launch_pdl(lora_project16_kernel<false>, dim3(grid), dim3(LP_THREADS), smem, s, js, n));
  }
  return launch_status("lora_project16_kernel launch");
}


// ---------------------------------------------------------------- weight grads
// G[r, c] = sum_t P[t, r] * Q[t, c] on the tensor cores: M = the 16 adapter rows, N = columns
// of Q, K = tokens.  Both operands are contiguous along M/N, not K, so each 32-token chunk of
// P and Q is staged in shared memory (cp.async, double-buffered) and the fragments are read
// with ldmatrix .trans.  A CTA of 4 warps owns 128 columns (32 per warp) of one token range
// ("split").  With one split the CTA writes its scaled result directly; otherwise it writes its
// fp32 partial to the workspace, takes a ticket on its column tile, and the tile's last CTA
// adds the partials up in split order (deterministic whatever the arrival order) and writes
// the result.  Nobody waits: each CTA publishes its partial before it takes its ticket, so the
// last ticket holder finds every partial in place.
constexpr int LO_THREADS = 128;
constexpr int LO_COLS = 128;                   // columns per CTA
constexpr int LO_TOK = 32;                     // tokens per staged chunk (two k16 steps)
constexpr int LO_STAGES = 4;                   // staged chunks in the ring
constexpr int LO_QROW = LO_COLS * 2 + 16;      // staged Q row, bytes (+16: conflict-free ldmatrix)
constexpr int LO_PROW = 48;                    // staged P row, bytes (32 of data + pad)
constexpr int LO_QBUF = LO_TOK * LO_QROW;
constexpr int LO_PBUF = LO_TOK * LO_PROW;
constexpr int LO_TARGET_CTAS = 2 * 148;        // two CTAs per SM of a B200, evenly
constexpr int LO_MIN_TOK = 64;                 // tokens per split at least (two chunks)
// Workspace: LO_CNT_BYTES of per-column-tile tickets (zero between calls; every call leaves
// them zero), then the fp32 partials [splits][16][cols] of each job with more than one split.
constexpr int LO_MAX_TILES = 1024;
constexpr int64_t LO_CNT_BYTES = LO_MAX_TILES * 4;

// One outer product of a launch: its CTAs are [cta0, cta0 + col tiles * splits), its tickets
// [tile0, tile0 + col tiles).
struct OuterJob {
  const __half* P;
  const __half* Q;
  float* partial;    // [splits][16][cols] (splits > 1)
  float* out;        // [16][cols], or [cols][16] when transpose
  int64_t cols;
  int64_t splits;
  int64_t tps;       // tokens per split
  float scale;
  int32_t transpose;
  int32_t cta0;
  int32_t tile0;
};
constexpr int LO_MAX_JOBS = 6;  // dA and dB of up to three adapters
struct OuterJobs {
  OuterJob j[LO_MAX_JOBS];
  int32_t* tickets;
  int32_t n;
};

__device__ __forceinline__ int find_job(const OuterJobs& js, int bid) {
  int k = 0;
  for (int i = 1; i < js.n; ++i)
    if (bid >= js.j[i].cta0) k = i;
  return k;
}

__global__ void __launch_bounds__(LO_THREADS)
    lora_grads16_kernel(const __grid_constant__ OuterJobs jobs, int64_t n) {
  grid_dep_wait();  // programmatic launch: no global access before the wait
  __shared__ __align__(128) uint8_t qbuf[LO_STAGES][LO_QBUF];
  __shared__ __align__(128) uint8_t pbuf[LO_STAGES][LO_PBUF];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const OuterJob& job = jobs.j[find_job(jobs, int(blockIdx.x))];
  const __half* __restrict__ P = job.P;
  const __half* __restrict__ Q = job.Q;
  const int64_t cols = job.cols;
  const int64_t col_tiles = (cols + LO_COLS - 1) / LO_COLS;
  const int64_t local = int64_t(blockIdx.x) - job.cta0;
  const int64_t split = local / col_tiles;
  const int64_t tile = local - split * col_tiles;
  const int64_t c0 = tile * LO_COLS;
  const int64_t tb = split * job.tps;
  const int64_t te = min64(n, tb + job.tps);

  // stage tokens [ts, ts + 32) of P (32 B per token) and of Q's 128 columns; rows past te or
  // columns past `cols` are zero-filled
  auto stage = [&](int buf, int64_t ts) {
    const uint32_t qb = smem_u32(qbuf[buf]), pb = smem_u32(pbuf[buf]);
#pragma unroll
    for (int i = 0; i < (LO_TOK * LO_COLS / 8) / LO_THREADS; ++i) {
      const int e = threadIdx.x + i * LO_THREADS;  // 16-byte piece: row e / 16, piece e % 16
      const int row = e >> 4, pc = e & 15;
      const int64_t t = ts + row, c = c0 + 8 * pc;
      const bool ok = t < te && c < cols;
      cp_async16(qb + row * LO_QROW + pc * 16, ok ? Q + t * cols + c : Q, ok);
    }
    if (threadIdx.x < LO_TOK * 2) {
      const int row = threadIdx.x >> 1, h = threadIdx.x & 1;
      const int64_t t = ts + row;
      cp_async16(pb + row * LO_PROW + h * 16, t < te ? P + t * 16 + 8 * h : P, t < te);
    }
    cp_async_commit();
  };

  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  // a ring of LO_STAGES chunk buffers: LO_STAGES - 1 chunks in flight while one is multiplied
  // (an empty commit group keeps the group count in step past the last chunk)
  const int64_t nchunks = (te - tb + LO_TOK - 1) / LO_TOK;
#pragma unroll
  for (int i = 0; i < LO_STAGES - 1; ++i) {
    if (i < nchunks)
      stage(i, tb + int64_t(i) * LO_TOK);
    else
      cp_async_commit();
  }
  for (int64_t ch = 0; ch < nchunks; ++ch) {
    const int buf = int(ch % LO_STAGES);
    cp_async_wait<LO_STAGES - 2>();  // chunk ch has landed
    __syncthreads();
    const uint32_t qb = smem_u32(qbuf[buf]), pb = smem_u32(pbuf[buf]);
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      // A[r][t] = P[t][r], stored [t][r]: matrices (r 0-7 | 8-15) x (t 0-7 | 8-15)
      uint32_t a[4];
      {
        const int j = lane >> 3, row = lane & 7;
        const int t = ks * 16 + (j >> 1) * 8 + row, r = (j & 1) * 8;
        ldsm_x4_t(pb + t * LO_PROW + r * 2, a);
      }
#pragma unroll
      for (int nt = 0; nt < 4; nt += 2) {
        // B[t][c] = Q[t][c], stored [t][c]: (t 0-7, t 8-15) for column tiles nt and nt+1
        uint32_t b[4];
        const int j = lane >> 3, row = lane & 7;
        const int t = ks * 16 + (j & 1) * 8 + row;
        const int col = 32 * warp + 8 * (nt + (j >> 1));
        ldsm_x4_t(qb + t * LO_QROW + col * 2, b);
        mma16816(acc[nt], a, b[0], b[1]);
        mma16816(acc[nt + 1], a, b[2], b[3]);
      }
    }
    __syncthreads();  // buffer `buf` is free: refill it with the chunk LO_STAGES - 1 ahead
    const int64_t nx = ch + LO_STAGES - 1;
    if (nx < nchunks)
      stage(int(nx % LO_STAGES), tb + nx * LO_TOK);
    else
      cp_async_commit();
  }
  cp_async_wait<0>();
  // D fragment: d[0..1] = G[g][2c..2c+1], d[2..3] = G[g+8][2c..2c+1] of each 16 x 8 tile
  const int g = lane >> 2, cq = lane & 3;
  const float scale = job.scale;
  float* __restrict__ out = job.out;
  if (job.splits == 1) {
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int64_t c = c0 + 32 * warp + 8 * nt + 2 * cq;
      if (c < cols) {
        if (job.transpose) {
          out[c * 16 + g] = acc[nt][0] * scale;
          out[(c + 1) * 16 + g] = acc[nt][1] * scale;
          out[c * 16 + g + 8] = acc[nt][2] * scale;
          out[(c + 1) * 16 + g + 8] = acc[nt][3] * scale;
        } else {
          *reinterpret_cast<float2*>(out + int64_t(g) * cols + c) = make_float2(acc[nt][0] * scale, acc[nt][1] * scale);
          *reinterpret_cast<float2*>(out + int64_t(g + 8) * cols + c) =
              make_float2(acc[nt][2] * scale, acc[nt][3] * scale);
        }
      }
    }
    return;
  }
  float* __restrict__ partial = job.partial;
  float* dst = partial + split * 16 * cols;
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const int64_t c = c0 + 32 * warp + 8 * nt + 2 * cq;
    if (c < cols) {
      __stcg(reinterpret_cast<float2*>(dst + int64_t(g) * cols + c), make_float2(acc[nt][0], acc[nt][1]));
      __stcg(reinterpret_cast<float2*>(dst + int64_t(g + 8) * cols + c), make_float2(acc[nt][2], acc[nt][3]));
    }
  }
  // publish the partial, then take the column tile's ticket
  __threadfence();
  __syncthreads();
  int32_t* ticket = jobs.tickets + job.tile0 + tile;
  if (threadIdx.x == 0) s_last = atomicAdd(ticket, 1) == int(job.splits) - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // the last CTA of the tile: column c0 + threadIdx.x, all 16 rows, splits in order
  const int64_t c = c0 + threadIdx.x;
  if (c < cols) {
    float sum[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) sum[r] = 0.f;
    for (int64_t sp = 0; sp < job.splits; ++sp) {
      const float* src = partial + sp * 16 * cols + c;
#pragma unroll
      for (int r = 0; r < 16; ++r) sum[r] += __ldcg(src + int64_t(r) * cols);
    }
    if (job.transpose) {
#pragma unroll
      for (int r = 0; r < 16; ++r) out[c * 16 + r] = sum[r] * scale;
    } else {
#pragma unroll
      for (int r = 0; r < 16; ++r) out[int64_t(r) * cols + c] = sum[r] * scale;
    }
  }
  if (threadIdx.x == 0) *ticket = 0;  // every CTA of the tile has taken its ticket: reset for reuse
}

// Splits (token ranges) of the jobs of one launch: at most LO_TARGET_CTAS CTAs over all the
// launch's column tiles (rounding down, so no SM gets a third CTA while others have two), at
// least LO_MIN_TOK tokens a split; one split when the tickets would not fit.
static int64_t grads_splits(int64_t n, int64_t col_tiles) {
  if (col_tiles > LO_MAX_TILES) return 1;
  int64_t s = LO_TARGET_CTAS / col_tiles;
  const int64_t max_s = (n + LO_MIN_TOK - 1) / LO_MIN_TOK;
  if (s > max_s) s = max_s;
  return s < 1 ? 1 : s;
}

// The launch of a list of outer products G = P^T Q over n tokens (scaled, optionally
// transposed): tickets and partials in `work` (LO_CNT_BYTES of zeroed tickets, then partials).
struct GradsPlan {
  OuterJobs js;
  int64_t ctas;
  int64_t bytes;  // workspace bytes the launch needs (0: no split)
};

struct GradsSpec {
  const __half* P;
  const __half* Q;
  int64_t cols;
  float scale;
  int transpose;
  float* out;
};

static GradsPlan plan_grads(const GradsSpec* specs, int n_specs, int64_t n, void* work) {
  GradsPlan p{};
  int64_t tiles = 0;
  for (int i = 0; i < n_specs; ++i) tiles += (specs[i].cols + LO_COLS - 1) / LO_COLS;
  const int64_t splits = grads_splits(n, tiles);
  float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(work) + LO_CNT_BYTES);
  int64_t floats = 0, ctas = 0, tile0 = 0;
  for (int i = 0; i < n_specs; ++i) {
    OuterJob& j = p.js.j[p.js.n++];
    const int64_t ct = (specs[i].cols + LO_COLS - 1) / LO_COLS;
    j.P = specs[i].P;
    j.Q = specs[i].Q;
    j.out = specs[i].out;
    j.cols = specs[i].cols;
    j.splits = splits;
    j.tps = (n + splits - 1) / splits;
    j.scale = specs[i].scale;
    j.transpose = specs[i].transpose;
    j.cta0 = int32_t(ctas);
    j.tile0 = int32_t(tile0);
    j.partial = splits > 1 && work ? part + floats : nullptr;
    if (splits > 1) floats += splits * 16 * specs[i].cols;
    ctas += splits * ct;
    tile0 += ct;
  }
  p.js.tickets = static_cast<int32_t*>(work);
  p.ctas = ctas;
  p.bytes = splits > 1 ? LO_CNT_BYTES + floats * int64_t(sizeof(float)) : 0;
  return p;
}

static int run_grads(const GradsPlan& p, int64_t n, cudaStream_t s) {
  NF4B_RETURN_IF(p.ctas > 0x7FFFFFFFll, NF4B_ERR_UNSUPPORTED);
  NF4B_CUDA_TRY(launch_pdl(lora_grads16_kernel, dim3(unsigned(p.ctas)), dim3(LO_THREADS), size_t(0), s, p.js, n));
  return launch_status("lora_grads16_kernel launch");
}

// dA = s (dY B)^T X and dB = s dY^T (X A^T) of one adapter, as two jobs of one launch.
static void adapter_specs(GradsSpec* sp, const __half* x, const __half* dy, const __half* xa,
                          const __half* dyb, float scale, float* da, float* db, int64_t in_f,
                          int64_t out_f) {
  sp[0] = GradsSpec{dyb, x, in_f, scale, 0, da};   // dA[r, i] = s * sum_t dyb[t, r] x[t, i]
  sp[1] = GradsSpec{xa, dy, out_f, scale, 1, db};  // dB[o, r] = s * sum_t dy[t, o] xa[t, r] (G^T)
}

}  // namespace nf4b

using namespace nf4b;

extern "C" int64_t nf4b_lora_grads_work_bytes(int64_t n, int64_t in_features, int64_t out_features,
                                              int32_t rank) {
  if (n < 0 || in_features <= 0 || out_features <= 0 || rank != 16) return -1;
  GradsSpec sp[2];
  adapter_specs(sp, nullptr, nullptr, nullptr, nullptr, 1.f, nullptr, nullptr, in_features, out_features);
  return plan_grads(sp, 2, n, nullptr).bytes;
}

// Shared checks of one adapter's operands.
static int check_adapter(const void* x, const void* dy, const void* xa, const void* dyb, const float* da,
                         const float* db, int64_t in_f, int64_t out_f) {
  NF4B_RETURN_IF(!x || !dy || !xa || !dyb || !da || !db, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(in_f <= 0 || out_f <= 0, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(in_f % 8 != 0 || out_f % 8 != 0, NF4B_ERR_UNSUPPORTED);
  NF4B_RETURN_IF(!aligned(x, 16) || !aligned(dy, 16) || !aligned(xa, 16) || !aligned(dyb, 16),
                 NF4B_ERR_ALIGNMENT);
  return NF4B_OK;
}

// Launches the grads of `n_specs` jobs with workspace `work` (work_bytes bytes; its ticket words
// zero), or zeros the outputs when there are no tokens.
static int launch_grads(const GradsSpec* sp, int n_specs, int64_t n, void* work, int64_t work_bytes,
                        cudaStream_t s) {
  if (n == 0) {
    for (int i = 0; i < n_specs; ++i)
      NF4B_CUDA_TRY(cudaMemsetAsync(sp[i].out, 0, size_t(16 * sp[i].cols) * sizeof(float), s));
    return NF4B_OK;
  }
  const GradsPlan p = plan_grads(sp, n_specs, n, work);
  NF4B_RETURN_IF(p.bytes > 0 && (!work || work_bytes < p.bytes), NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(p.bytes > 0 && !aligned(work, 256), NF4B_ERR_ALIGNMENT);
  return run_grads(p, n, s);
}

extern "C" int nf4b_lora_grads(const void* x, const void* dy, const void* xa, const void* dyb,
                               float scale, float* da, float* db, void* work, int64_t n,
                               int64_t in_features, int64_t out_features, int32_t rank,
                               void* stream) {
  NF4B_RETURN_IF(n < 0, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(rank != 16, NF4B_ERR_UNSUPPORTED);
  int st = check_adapter(x, dy, xa, dyb, da, db, in_features, out_features);
  if (st != NF4B_OK) return st;
  st = check_device();
  if (st != NF4B_OK) return st;
  GradsSpec sp[2];
  adapter_specs(sp, static_cast<const __half*>(x), static_cast<const __half*>(dy),
                static_cast<const __half*>(xa), static_cast<const __half*>(dyb), scale, da, db, in_features,
                out_features);
  const int64_t need = plan_grads(sp, 2, n, nullptr).bytes;
  return launch_grads(sp, 2, n, work, need, static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------- several adapters in one launch
extern "C" int64_t nf4b_lora_grads_group_work_bytes(const nf4b_lora_grads_item* items, int32_t n_items,
                                                    int64_t n) {
  if (!items || n_items < 1 || n_items > LO_MAX_JOBS / 2 || n < 0) return -1;
  GradsSpec sp[LO_MAX_JOBS];
  for (int i = 0; i < n_items; ++i) {
    if (items[i].in_features <= 0 || items[i].out_features <= 0) return -1;
    adapter_specs(sp + 2 * i, nullptr, nullptr, nullptr, nullptr, 1.f, nullptr, nullptr, items[i].in_features,
                  items[i].out_features);
  }
  return plan_grads(sp, 2 * n_items, n, nullptr).bytes;
}

extern "C" int nf4b_lora_grads_group(const nf4b_lora_grads_item* items, int32_t n_items, void* work,
                                     int64_t work_bytes, int64_t n, void* stream) {
  NF4B_RETURN_IF(!items || n_items < 1 || n < 0, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(n_items > LO_MAX_JOBS / 2, NF4B_ERR_UNSUPPORTED);
  GradsSpec sp[LO_MAX_JOBS];
  for (int i = 0; i < n_items; ++i) {
    const nf4b_lora_grads_item& it = items[i];
    const int st = check_adapter(it.x, it.dy, it.xa, it.dyb, it.da, it.db, it.in_features, it.out_features);
    if (st != NF4B_OK) return st;
    adapter_specs(sp + 2 * i, static_cast<const __half*>(it.x), static_cast<const __half*>(it.dy),
                  static_cast<const __half*>(it.xa), static_cast<const __half*>(it.dyb), it.scale, it.da, it.db,
                  it.in_features, it.out_features);
  }
  const int st = check_device();
  if (st != NF4B_OK) return st;
  return launch_grads(sp, 2 * n_items, n, work, work_bytes, static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------- entry point without allocation
// For callers that cannot call cudaMalloc on this path -- code running inside a framework that
// has already reserved the device's memory for its own pool (an allocation behind its back can
// fail or break its accounting), or a latency-critical loop where allocating is not allowed --
// nf4b_lora_grads_noalloc keeps its split-token partial sums in this fixed file-scope device
// array instead of a caller-provided buffer.  Every GPU that loads the library holds these
// NF4B_NOALLOC_SCRATCH_BYTES until the process exits.  All calls share it: calls that overlap on
// the GPU (other streams, other host threads) race on it.  Its leading ticket words are zero when
// the library is loaded (a __device__ array starts zeroed) and every call leaves them zero; each
// call writes every partial sum it later reads, so nothing else has to start at zero.
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
  NF4B_RETURN_IF(n < 0, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(rank != 16, NF4B_ERR_UNSUPPORTED);
  int st = check_adapter(x, dy, xa, dyb, da, db, in_features, out_features);
  if (st != NF4B_OK) return st;
  const int64_t need = nf4b_lora_grads_work_bytes(n, in_features, out_features, rank);
  if (need > int64_t(NF4B_NOALLOC_SCRATCH_BYTES)) {
    record_message("nf4b_lora_grads_noalloc: the split-token partial sums need more than "
                   "NF4B_NOALLOC_SCRATCH_BYTES; use nf4b_lora_grads with a caller buffer");
    return NF4B_ERR_UNSUPPORTED;
  }
  st = check_device();
  if (st != NF4B_OK) return st;
  float* work = nullptr;
  st = noalloc_scratch(&work);
  if (st != NF4B_OK) return st;
  GradsSpec sp[2];
  adapter_specs(sp, static_cast<const __half*>(x), static_cast<const __half*>(dy),
                static_cast<const __half*>(xa), static_cast<const __half*>(dyb), scale, da, db, in_features,
                out_features);
  return launch_grads(sp, 2, n, work, NF4B_NOALLOC_SCRATCH_BYTES, static_cast<cudaStream_t>(stream));
}
