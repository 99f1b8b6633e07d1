// Fused NF4 dequant + GEMM on the 5th-gen tensor cores (tcgen05, TMEM, TMA).
//
// Forward  (patched MatMul4Bit.forward, solution/nf4.py:142-159 = unpack + F.linear):
//     Y[n, out]  = X[n, in] . W[out, in]^T (+ bias) (+ (X A^T) (s B)^T)
// Backward (bitsandbytes MatMul4Bit.backward grad_A on the re-unpacked weight):
//     dX[n, in]  = dY[n, out] . W[out, in] (+ (dY B) (s A))
//
// Both are computed transposed on the tensor core ("swap AB"): the MMA's M side is
// the weight (128 rows = out features forward, in features backward) and its N side
// is up to 256 tokens, so a decoded 128 x 64 weight tile feeds 128x256x64 MACs.
//   D[m, t] (TMEM, fp32) = sum_k Wtile[m, k] . Act[t, k]
//
// Persistent, warp-specialised: one CTA per SM walks output tiles (128 weight rows x
// 256 tokens) with stride gridDim.x; the 4-stage shared-memory ring and the stage
// counters run on across tiles, and the two 256-column accumulators in TMEM alternate
// between tiles, so a tile's epilogue overlaps the next tile's main loop.
// Pairs (PAIR): 2-CTA clusters walk 256-row x 512-token tiles; each decoded weight stage
// feeds two cta_group::2 MMAs (tokens [0, 256) and [256, 512) of the tile), halving the
// decode per FLOP, into one 512-column accumulator that the epilogue drains in halves.
//   warp 0      TMA producer: activation tile [256 tok x 64] fp16 (128B swizzle) and
//               the packed weight tile (4 KB) per stage.
//   warp 1      TMEM allocation (512 columns) + single-thread tcgen05.mma issuer.
//   warps 2-9   decode the packed tile in registers (nf4_decode.cuh) straight into the
//               128B-swizzled fp16 operand layout (K-major forward, MN-major backward).
//   warps 10-17 epilogue: tcgen05.ld of the finished accumulator -> fp16 -> global.
// LoRA is one extra K=16 MMA ("slab") into the tile's accumulator (a pair tile: one per
// token half): the rank-16 token activations (X A^T or dY B, from lora.cu) against the scaled
// adapter weight.
//
// Every pipeline wait is bounded (~2 s); on expiry the CTA raises an abort flag,
// records the failure in g_gemm_error, and winds down without hanging the GPU.
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "nf4_decode.cuh"

namespace nf4b {

constexpr int G_M = 128;       // MMA M: weight rows per tile
constexpr int G_NMAX = 256;    // MMA N: tokens per tile
constexpr int G_K = 64;        // K per pipeline stage (one 128-byte swizzle row of fp16)
constexpr int G_DQ_WARPS = 8;
constexpr int G_EPI_WARPS = 8;
constexpr int G_DQ_WARP0 = 2;
constexpr int G_EPI_WARP0 = G_DQ_WARP0 + G_DQ_WARPS;  // 10
constexpr int G_THREADS = 32 * (G_EPI_WARP0 + G_EPI_WARPS);
constexpr int G_ACC_COLS = 256;                        // one accumulator
constexpr int G_TMEM_COLS = 2 * G_ACC_COLS;            // double-buffered

constexpr int G_MAX_W = 3;  // NF4 weights of one grouped forward launch

// Tokens of a pair tile: two cta_group::2 MMAs of up to 256 tokens each share one decoded
// weight stage, so a pair decodes each weight stage once per 512 tokens.
constexpr int G_PAIR_TILE_N = 2 * G_NMAX;

// Shared-memory layout of one CTA.  PAIR: the CTA is half of a 2-CTA cluster whose two MMAs
// (cta_group::2) cover 256 weight rows x up to 2 x 256 tokens; each CTA holds its own 128
// decoded weight rows and, per MMA, half of its tokens (two 128-row halves per stage).
template <bool PAIR>
struct Smem {
  static constexpr int STAGES = 4;
  static constexpr int X_ROWS = G_NMAX;                      // token rows per CTA and stage
  static constexpr int X_BYTES = X_ROWS * 128;               // activation stage
  static constexpr int A_BYTES = G_M * 128;                  // decoded weight stage
  static constexpr int P_BYTES = 4096;                       // packed stage (128 x 32 B or 64 x 64 B)
  static constexpr int LA_BYTES = G_M * 32;                  // LoRA slab, weight side [128][16] fp16
  static constexpr int LB_BYTES = X_ROWS * 32;               // LoRA slab, token side [rows][16] fp16
  static constexpr int X = 0;
  static constexpr int A = X + STAGES * X_BYTES;
  static constexpr int P = A + STAGES * A_BYTES;
  static constexpr int LA = P + STAGES * P_BYTES;
  static constexpr int LB = LA + LA_BYTES;
  static constexpr int CODE = LB + LB_BYTES;         // per weight: 16 fp32 NF4 code
  static constexpr int CODE2 = CODE + 64 * G_MAX_W;  // per weight: 256 fp32 second-level code
  static constexpr int BAR = CODE2 + 1024 * G_MAX_W;
  // full[S], afull[S], empty[S], acc_full[2], acc_empty[2], lora_full, lora_empty, mma_done,
  // red_full[2] (split-K partials staged into the idle ring, RED_* below)
  static constexpr int NUM_BARS = 3 * STAGES + 9;
  static constexpr int MISC = BAR + NUM_BARS * 8;
  static constexpr int WU0 = MISC + 16;  // the CTA's first work unit, computed in the prologue
  static constexpr int TOTAL = WU0 + 64;
  static constexpr int ALLOC = TOTAL + 1024;  // slack to align the base to 1024 B
  // Split-K reduction of a CTA's last work unit: the activation and decoded-weight stages
  // (contiguous from offset 0) are idle once that unit's accumulator is complete, and hold
  // two rounds x RED_PARTS slices of 64 tokens x 128 rows fp32 (32 KB) of the other ranges'
  // partial tiles.
  static constexpr int RED_SLICE = 64 * G_M * 4;
  static constexpr int RED_PARTS = (X + STAGES * (X_BYTES + A_BYTES)) / (2 * RED_SLICE);
};
static_assert(Smem<false>::ALLOC <= 232448 && Smem<true>::ALLOC <= 232448, "shared memory budget");

// Split-K workspace: a fixed counter region (arrivals at [0, G_SPLIT_MAX_TILES), finished
// partials at [G_SPLIT_MAX_TILES, 2 * G_SPLIT_MAX_TILES), the launch's exit count at
// G_SPLIT_EXIT, padded to 256 B so the partial tiles keep whole 128-byte lines), then the
// fp32 partial tiles.  The region does not depend on the launch's shape, so one zeroed
// workspace serves any sequence of calls on a stream: the last CTA to leave a launch clears
// every counter the launch used, also when a range gave up before taking its ticket.
constexpr int G_SPLIT_MAX_TILES = 512;
constexpr int G_SPLIT_EXIT = 2 * G_SPLIT_MAX_TILES;
// Tokens of one CTA's fp32 partial tile: the accumulator columns of a tile.
template <bool PAIR>
constexpr int acc_tokens() { return PAIR ? G_PAIR_TILE_N : G_ACC_COLS; }
constexpr int64_t G_SPLIT_CNT_BYTES = 2 * G_SPLIT_MAX_TILES * 4 + 256;

// One NF4 weight of a launch.  A forward launch may carry up to G_MAX_W weights that share
// the activation X (q/k/v, gate/up): their 128-row tiles are numbered one after the other.
struct GemmW {
  const uint8_t* absmax8;
  const float* absmax32;
  const float* code2;
  const float* absmax2;
  const float* offset;
  const float* code;
  const __half* bias;     // forward only, [out] or null
  const __half* lora_w;   // forward: lora B [out, 16]; backward: lora A [16, in]
  const __half* lora_t;   // forward: X A^T [n, 16];   backward: dY B [n, 16]
  __half* out;            // forward: Y [n, out]; backward: dX [n, in]
  int64_t out_f;          // out features of this weight
  float lora_scale;
  int32_t has_lora;
  int32_t log2_bs;
  int32_t nested;
};

struct GemmArgs {
  GemmW w[G_MAX_W];
  int32_t nw;             // weights in use
  int32_t m_end[G_MAX_W]; // forward: weight i owns global 128-row tiles [m_end[i-1], m_end[i])
  int32_t k_end[G_MAX_W]; // backward: weight i owns K stages [k_end[i-1], k_end[i]) (its out features)
  int64_t n;
  int64_t in_f;
  int32_t m_tiles;        // 128-row weight tiles, all weights
  int32_t n_tiles;        // 256-token tiles
  int32_t splits;         // K ranges per tile (split-K); 1 = none
  int32_t nk;             // K stages of the whole reduction
  uint32_t k16;           // 1 << 16 (a run-time multiplier for the decode's shifts)
  int32_t tile_n;         // tokens per tile: 256 or 128 (single CTAs), 512 (pairs)
  float* ws_part;         // split-K: fp32 partial tiles [tiles][splits][256][128]
  int32_t* ws_cnt;        // split-K: per-tile counters [2][G_SPLIT_MAX_TILES] + exit count, zero
                          // between launches
  int32_t drop_ticket_unit;  // test hook: this work unit skips its ticket (-1: none)
  int32_t epi_decode;     // a backward launch whose CTAs (pairs) have at most one work unit: the
                          // epilogue warps decode stages too until their accumulator is ready
  __half* glu_out;        // SwiGLU launches: m = fp16(gate * sigmoid(gate) * up) [n, out]
  int32_t red_staged;     // split-K: the last range of a tile reads the other ranges' partials
                          // through bulk copies into the idle ring (its CTA's last unit only)
  // SwiGLU-backward launches (dX of down): the forward's gate and up [n, in], and the outputs
  // dgate, dup [n, in] written instead of dX
  const __half* glu_g;
  const __half* glu_u;
  __half* glu_dg;
  __half* glu_du;
};

__device__ int g_gemm_error;

constexpr long long kWaitLimitCycles = 4000000000ll;  // ~2 s at 1.9 GHz

// Longest time a waiting thread stays suspended in one try_wait: waiting warps sleep in
// hardware until the phase completes instead of spinning on issue slots that the decode
// warps need, and still look at the abort flag and the clock about once a millisecond.
constexpr uint32_t kSuspendHintNs = 1000000u;

// Bounded pipeline wait.  On expiry the abort flag of this CTA and, through `peer_abort` (a
// shared::cluster address, 0 for none), that of the other CTA of a pair are raised.
__device__ __forceinline__ bool pipe_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          uint32_t peer_abort) {
  // a phase that has already completed (the MMA issuer's usual case) is seen without the
  // suspend/resume cost of try_wait
  if (mbar_test_wait(bar, parity)) return true;
  if (mbar_try_wait_sleep(bar, parity, kSuspendHintNs)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitLimitCycles) {
      *abort_flag = 1;
      if (peer_abort) st_cluster_u32(peer_abort, 1u);
      atomicExch(&g_gemm_error, 1);
      return false;
    }
    if (mbar_try_wait_sleep(bar, parity, kSuspendHintNs)) return true;
  }
}

// Time-bounded wait that ignores the abort flag (used to drain in-flight work).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait_sleep(bar, parity, kSuspendHintNs)) {
    if (clock64() - t0 > kWaitLimitCycles) {
      atomicExch(&g_gemm_error, 2);
      return;
    }
  }
}

// SWIZZLE_NONE K-major descriptor: 8-row x 16-byte core matrices; K-adjacent core
// matrices `lbo` apart, 8-row groups `sbo` apart.
__device__ __forceinline__ uint64_t smem_desc_nosw(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3FFF);
  d |= uint64_t((lbo >> 4) & 0x3FFF) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFF) << 32;
  d |= uint64_t(1) << 46;
  return d;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// Byte offset of LoRA slab element row `r`, 16-byte chunk `kc` (0/1): [r/8][kc][r%8][16 B].
__device__ __forceinline__ uint32_t slab_off(int r, int kc) {
  return uint32_t((r >> 3) * 256 + kc * 128 + (r & 7) * 16);
}

// sigmoid of the SwiGLU epilogue: fast exp and divide, the expression of the standalone SwiGLU
// kernel (step_ops.cu) -- m = fp16(g * sigmoid(g) * u) with fp32 inside, the rounding points
// of the reference's SwiGLU kernel (solution/swiglu.py:16-23).  (The IEEE-exact exp and divide
// cost the epilogue enough issue slots to slow the decode: 96.4 vs 76.7 us on gate/up at 1,170
// tokens.)
__device__ __forceinline__ float glu_sigmoid(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

__device__ __forceinline__ uint4 scale_pack8(uint4 v, float s) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
  uint4 o;
  uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    op[i] = pack_half2(f.x * s, f.y * s);
  }
  return o;
}

struct ScaleSrc {
  uint32_t q;   // nested: 8-bit code
  float a;      // nested: second-level absmax; plain: absmax
};

__device__ __forceinline__ ScaleSrc load_scale_src(const GemmW& W, int64_t blk, bool valid) {
  ScaleSrc s{0u, 0.f};
  if (!valid) return s;
  if (W.nested) {
    s.q = __ldg(W.absmax8 + blk);
    s.a = __ldg(W.absmax2 + (blk >> 8));
  } else {
    s.a = __ldg(W.absmax32 + blk);
  }
  return s;
}

struct TileCoord {
  int seg;      // weight of the tile (index into GemmArgs::w)
  int64_t m0;   // first row of that weight (forward: out feature; backward: in feature)
  int64_t t0;   // first token
  int tn_real;  // tokens in this tile
  int tn;       // MMA N (tn_real rounded up to 16)
};

// MULTI: the launch carries more than one weight (a grouped forward).  Single-weight launches
// compile with the weight index fixed at 0, so its fields stay direct constant-bank operands.
// PAIR: tiles are 256 weight rows, of which CTA `rank` of the pair owns rows 128 rank ..
// GLU: a SwiGLU forward launch over gate (weight 0) and up (weight 1): a CTA's 128 rows are 64 features
// of both, so m0 is the first of the CTA's 64 features.
template <bool MULTI, bool PAIR, bool GLU>
__device__ __forceinline__ TileCoord tile_coord(const GemmArgs& g, int tile, uint32_t rank) {
  TileCoord c;
  const int mt = tile / g.n_tiles;
  const int nt = tile - mt * g.n_tiles;
  c.seg = MULTI ? (mt >= g.m_end[0]) + (mt >= g.m_end[1]) : 0;
  c.m0 = GLU ? int64_t(mt) * (PAIR ? G_M : G_M / 2) + int64_t(rank) * (G_M / 2)
             : int64_t(mt - (c.seg ? g.m_end[c.seg - 1] : 0)) * (PAIR ? 2 * G_M : G_M) + int64_t(rank) * G_M;
  c.t0 = int64_t(nt) * g.tile_n;
  c.tn_real = int(min64(g.tile_n, g.n - c.t0));
  c.tn = (c.tn_real + 15) & ~15;
  return c;
}

// Work unit of the persistent loop: one K range of one output tile.  The units of a tile
// are consecutive, so its K ranges run at the same time on neighbouring CTAs.
struct WorkUnit {
  TileCoord tc;
  int tile;
  int split;
  int kb, ke;   // stage range [kb, ke)
};

static_assert(sizeof(WorkUnit) <= 64, "the prologue keeps one WorkUnit in 64 bytes of shared memory");

template <bool MULTI, bool PAIR, bool GLU>
__device__ __forceinline__ WorkUnit work_unit(const GemmArgs& g, int u, uint32_t rank) {
  WorkUnit w;
  w.tile = u / g.splits;
  w.split = u - w.tile * g.splits;
  w.tc = tile_coord<MULTI, PAIR, GLU>(g, w.tile, rank);
  w.kb = (w.split * g.nk) / g.splits;  // splits <= 8, so 32 bits hold the products
  w.ke = ((w.split + 1) * g.nk) / g.splits;
  return w;
}

// 32 lanes x 16 columns of fp32 from TMEM (thread t: row lane base + t, columns [col, col+16)).
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// A backward launch over several weights concatenates their K (each weight's out features):
// stage k belongs to weight kseg(k), whose local stage is k - kbeg(kseg(k)).
__device__ __forceinline__ int kseg(const GemmArgs& g, int k) {
  return (k >= g.k_end[0]) + (k >= g.k_end[1]);
}
__device__ __forceinline__ int kbeg(const GemmArgs& g, int s) { return s ? g.k_end[s - 1] : 0; }

// Named barrier 1 over the epilogue warps only.
__device__ __forceinline__ void epi_bar_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(G_EPI_WARPS * 32) : "memory");
}
// Same barrier, returning the AND of `v` over the epilogue threads.
__device__ __forceinline__ bool epi_bar_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(v)), "n"(G_EPI_WARPS * 32)
      : "memory");
  return r != 0;
}

// Bounded wait until *p == want (acquire at GPU scope); false on timeout.
__device__ __forceinline__ bool wait_count(const int32_t* p, int want) {
  const long long t0 = clock64();
  for (;;) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    if (v == want) return true;
    if (clock64() - t0 > kWaitLimitCycles) {
      atomicExch(&g_gemm_error, 3);
      return false;
    }
    __nanosleep(64);
  }
}

// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from global memory
// into this CTA's shared memory, completing on mbarrier `bar` (no multicast).
__device__ __forceinline__ void bulk_load_g2s(uint32_t smem_dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
// Orders this thread's earlier generic-proxy accesses of global memory (here: an acquire of
// the partial tiles' arrival count) before its later async-proxy ones (the bulk copies).
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// SPLIT: compiled with the split-K epilogue (launches with g.splits > 1).
// PAIR: launched as 2-CTA clusters; CTA rank 0 issues cta_group::2 MMAs over both CTAs' tiles.
// GLU, forward: the SwiGLU forward of an MLP: gate and up in one tile, epilogue writes gate, up
// and m = fp16(gate * sigmoid(gate) * up).  GLU, backward: dX of the MLP's down projection, whose
// epilogue applies the SwiGLU backward (dgate, dup from dm = the rounded dX and the forward's
// gate and up) instead of writing dm.
template <bool BWD, bool SPLIT, bool MULTI, bool PAIR, bool GLU>
__global__ void __launch_bounds__(G_THREADS, 1)
    nf4_gemm_kernel(const __grid_constant__ CUtensorMap tm_act0, const __grid_constant__ CUtensorMap tm_act1,
                    const __grid_constant__ CUtensorMap tm_act2, const __grid_constant__ CUtensorMap tm_w0,
                    const __grid_constant__ CUtensorMap tm_w1, const __grid_constant__ CUtensorMap tm_w2,
                    const __grid_constant__ GemmArgs g) {
  // BWD && MULTI: several weights along K (dX = sum_i dY_i W_i); !BWD && MULTI: several
  // weights along M (Y_i = X W_i^T).
  constexpr bool KCAT = BWD && MULTI;
  static_assert(!GLU || !MULTI, "SwiGLU launches carry one gate/up pair (forward) or down (backward)");
  constexpr bool GLUF = GLU && !BWD;  // SwiGLU forward tiles (gate and up rows side by side)
  using L = Smem<PAIR>;
  constexpr int NS = L::STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint64_t* afull = full + NS;
  uint64_t* empty = afull + NS;
  uint64_t* acc_full = empty + NS;        // [2]
  uint64_t* acc_empty = acc_full + 2;     // [2]
  uint64_t* lora_full = acc_empty + 2;
  uint64_t* lora_empty = lora_full + 1;
  uint64_t* mma_done = lora_empty + 1;
  uint64_t* red_full = mma_done + 1;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC + 4);
  float* s_code = reinterpret_cast<float*>(smem + L::CODE);
  float* s_code2 = reinterpret_cast<float*>(smem + L::CODE2);

  const int nunits = g.m_tiles * g.n_tiles * g.splits;
  // PAIR: this CTA's rank in its cluster, the cluster's index, and the barriers of rank 0
  // (the MMA issuer) that both CTAs arrive on, as shared::cluster addresses.
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int unit0 = PAIR ? int(cluster_id_x()) : int(blockIdx.x);
  const int ustride = PAIR ? int(cluster_count_x()) : int(gridDim.x);
  const uint32_t peer_abort = PAIR ? mapa_shared(smem_u32((const void*)abort_flag), rank ^ 1u) : 0u;
  const uint32_t afull_l = PAIR ? mapa_shared(smem_u32(afull), 0u) : smem_u32(afull);
  const uint32_t acc_empty_l = PAIR ? mapa_shared(smem_u32(acc_empty), 0u) : smem_u32(acc_empty);
  const uint32_t lora_full_l = PAIR ? mapa_shared(smem_u32(lora_full), 0u) : smem_u32(lora_full);
  auto pwait = [&](uint64_t* bar, uint32_t ph) { return pipe_wait(bar, ph, abort_flag, peer_abort); };
  // arrival (one per warp) on a barrier that the MMA issuer waits on: `bar` is this CTA's
  // copy, `bar_l` the issuer's copy as a shared::cluster address
  auto arrive_issuer = [&](uint64_t* bar, uint32_t bar_l) {
    if (PAIR)
      mbar_arrive_cl(bar_l);
    else
      mbar_arrive(bar);
  };
  // MMA completion -> barrier `bar` of this CTA and, for a pair, the same barrier of rank 1
  auto commit_both = [&](uint64_t* bar) {
    if (PAIR) {
      umma_commit_pair(smem_u32(bar));
      umma_commit_pair(mapa_shared(smem_u32(bar), 1u));
    } else {
      umma_commit(bar);
    }
  };
  constexpr uint32_t kPeers = PAIR ? 2u : 1u;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&afull[i], kPeers * (G_DQ_WARPS / 2));
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kPeers * G_EPI_WARPS);
    }
    mbar_init(lora_full, kPeers * G_DQ_WARPS);
    mbar_init(lora_empty, 1);
    mbar_init(mma_done, 1);
    mbar_init(&red_full[0], 1);
    mbar_init(&red_full[1], 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tma_desc(&tm_act0);
    prefetch_tma_desc(&tm_w0);
    if (g.nw > 1) prefetch_tma_desc(&tm_w1);
    if (g.nw > 2) prefetch_tma_desc(&tm_w2);
    if (KCAT && g.nw > 1) prefetch_tma_desc(&tm_act1);
    if (KCAT && g.nw > 2) prefetch_tma_desc(&tm_act2);
    // the first work unit, for every role: its kernel-parameter reads (a chain of constant-cache
    // misses on a cold SM) happen here, before the programmatic-launch wait, instead of in front
    // of the first bulk copy
    *reinterpret_cast<WorkUnit*>(smem + L::WU0) = work_unit<MULTI, PAIR, GLUF>(g, unit0 < nunits ? unit0 : 0, rank);
  }
  const WorkUnit& wu_first = *reinterpret_cast<const WorkUnit*>(smem + L::WU0);
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(tmem_slot, G_TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, G_TMEM_COLS);
      tmem_relinquish();
    }
  }
  // everything above overlaps the previous kernel of the stream (programmatic launch); global
  // memory is touched only after it has completed
  grid_dep_wait();
  for (int i = 0; i < g.nw; ++i) {
    if (threadIdx.x < 16) s_code[16 * i + threadIdx.x] = __ldg(g.w[i].code + threadIdx.x);
    if (g.w[i].nested && threadIdx.x < 256) s_code2[256 * i + threadIdx.x] = __ldg(g.w[i].code2 + threadIdx.x);
  }
  tc_fence_before();
  __syncthreads();
  // a pair: both CTAs' barriers initialised and TMEM allocated before any remote arrival/MMA
  if (PAIR) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int u = unit0; ok && u < nunits; u += ustride) {
        const WorkUnit wu = u == unit0 ? wu_first : work_unit<MULTI, PAIR, GLUF>(g, u, rank);
        const TileCoord& tc = wu.tc;
        // A pair tile's MMA h (h = 0, 1) covers tokens [256 h, 256 h + n_h) of the tile, n_h =
        // min(tn - 256 h, 256); it reads the first n_h / 2 of them from rank 0 and the rest
        // from rank 1, as one 128-row box per half and CTA.
        const int nh = (PAIR && tc.tn > G_NMAX) ? 2 : 1;
        int trow[2];
        for (int h = 0; h < 2; ++h)
          trow[h] = int(tc.t0) + (PAIR ? h * G_NMAX + int(rank) * (min(tc.tn - h * G_NMAX, G_NMAX) >> 1) : 0);
        for (int k = wu.kb; k < wu.ke; ++k, ++it) {
          const int s = it % NS;
          const uint32_t ph = (it / NS) & 1;
          if (!pwait(&empty[s], ph ^ 1)) {
            ok = false;
            break;
          }
          // the token box is the tile width (a pair: one 128-row box per MMA)
          mbar_arrive_expect_tx(&full[s], (PAIR ? nh * (G_NMAX / 2) * 128 : g.tile_n * 128) + L::P_BYTES);
          const int ws = KCAT ? kseg(g, k) : tc.seg;   // weight of this stage
          const int kl = KCAT ? k - kbeg(g, ws) : k;  // its local K stage
          const CUtensorMap* tm_a = ws == 0 ? &tm_act0 : (ws == 1 ? &tm_act1 : &tm_act2);
          const CUtensorMap* tm_w = ws == 0 ? &tm_w0 : (ws == 1 ? &tm_w1 : &tm_w2);
          for (int h = 0; h < nh; ++h)
            tma_load_2d(smem + L::X + s * L::X_BYTES + h * (G_NMAX / 2) * 128, KCAT ? tm_a : &tm_act0,
                        &full[s], kl * G_K, trow[h]);
          if (GLUF) {
            // gate rows [m0, m0 + 64) in packed rows 0-63, up rows [m0, m0 + 64) in rows 64-127
            tma_load_2d(smem + L::P + s * L::P_BYTES, &tm_w0, &full[s], kl * (G_K / 2), int(tc.m0));
            tma_load_2d(smem + L::P + s * L::P_BYTES + L::P_BYTES / 2, &tm_w1, &full[s], kl * (G_K / 2),
                        int(tc.m0));
          } else if (!BWD)
            tma_load_2d(smem + L::P + s * L::P_BYTES, tm_w, &full[s], kl * (G_K / 2), int(tc.m0));
          else
            tma_load_2d(smem + L::P + s * L::P_BYTES, tm_w, &full[s], int(tc.m0 / 2), kl * G_K);
        }
      }
      // no bulk copy may still be landing in this CTA's shared memory at exit
      for (uint32_t j = (it > uint32_t(NS) ? it - NS : 0); j < it; ++j)
        drain_wait(&full[j % NS], (j / NS) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    // (a pair: rank 0 issues for both CTAs; rank 1 only waits for the last MMA before its
    // TMEM is released)
    if (lane == 0 && rank == 0) {
      uint32_t it = 0, lt = 0, lc = 0;
      bool ok = true;
      const uint64_t ad0 = BWD ? smem_desc_sw128(sbase + L::A, 8192, 1024) : smem_desc_sw128(sbase + L::A, 16, 1024);
      const uint64_t bd0 = smem_desc_sw128(sbase + L::X, 16, 1024);
      for (int u = unit0; ok && u < nunits; u += ustride, ++lt) {
        const WorkUnit wu = u == unit0 ? wu_first : work_unit<MULTI, PAIR, GLUF>(g, u, rank);
        const TileCoord& tc = wu.tc;
        // Single CTAs: one 256-column accumulator per tile, two alternating between tiles
        // (acc_full / acc_empty[b]).  Pairs: one 512-column accumulator per tile, MMA h writing
        // columns [256 h, 256 h + n_h) (token 256 h + c of the tile); acc_full / acc_empty[h]
        // hand half h to the epilogue and back, so the drain of half 0 overlaps the tile's last
        // half-1 MMAs and the next tile's half-0 MMAs overlap the drain of half 1.
        const uint32_t b = PAIR ? 0u : (lt & 1);
        const uint32_t epar = PAIR ? ((lt & 1) ^ 1) : (((lt >> 1) & 1) ^ 1);
        const int n0 = PAIR ? min(tc.tn, G_NMAX) : tc.tn;
        const int n1 = PAIR ? tc.tn - n0 : 0;
        constexpr int MM = PAIR ? 2 * G_M : G_M;
        const uint32_t d0 = tmem_base + b * G_ACC_COLS;
        const uint32_t d1 = tmem_base + G_NMAX;
        const uint32_t id0 = idesc_f16(MM, n0, BWD, false);
        const uint32_t id1 = idesc_f16(MM, n1 > 0 ? n1 : 16, BWD, false);
        if (!pwait(&acc_empty[b], epar)) break;
        // a pair's half 1 is awaited before its first MMA (or, when the tile has no half-1
        // tokens, before acc_full[1] is committed, so that barrier never runs two phases ahead
        // of the epilogue)
        bool free1 = !PAIR;
        auto take1 = [&]() -> bool {
          if (!free1) free1 = pwait(&acc_empty[1], epar);
          return free1;
        };
        auto mma = [&](uint32_t d, uint64_t a, uint64_t bd, uint32_t id, bool accum) {
          if (PAIR)
            umma_f16_pair(d, a, bd, id, accum ? 1u : 0u);
          else
            umma_f16(d, a, bd, id, accum ? 1u : 0u);
        };
        tc_fence_after();
        bool acc0 = false, acc1 = false;
        // LoRA terms belong to the first K range; a K-concatenated backward has one slab per
        // adapter, filled and consumed one after the other
        for (int i = 0; wu.split == 0 && i < (KCAT ? g.nw : 1); ++i) {
          if (!g.w[KCAT ? i : (MULTI ? tc.seg : 0)].has_lora) continue;
          if (!pwait(lora_full, lc & 1)) {
            ok = false;
            break;
          }
          ++lc;
          tc_fence_after();
          const uint64_t ad = smem_desc_nosw(sbase + L::LA, 128, 256);
          const uint64_t bd = smem_desc_nosw(sbase + L::LB, 128, 256);
          mma(d0, ad, bd, idesc_f16(MM, n0, false, false), acc0);
          acc0 = true;
          if (PAIR && n1 > 0) {
            if (!take1()) {
              ok = false;
              break;
            }
            tc_fence_after();
            // the slab's token rows of half 1 start at row 128 (4 KB)
            mma(d1, ad, bd + uint64_t(4096 >> 4), idesc_f16(MM, n1, false, false), acc1);
            acc1 = true;
          }
          commit_both(lora_empty);
        }
        if (!ok) break;
        // The issuing thread shares its SM sub-partition with decode warps, so its loop is
        // kept short: afull alone is awaited (every decode warp arrives only after its own
        // full[s], so the stage's tokens have landed too -- for a pair, rank 1's half as
        // well), and the descriptors are slot-0 descriptors plus constant offsets (the ring
        // lies below 256 KB, so the 14-bit address field of a descriptor never carries).
        // The next stage's barrier is tested (without blocking) between this stage's MMAs, so
        // that test overlaps their issue and a ready stage follows without a wait.
        uint32_t s = it % NS, ph = (it / NS) & 1;
        bool ready = wu.kb < wu.ke && pwait(&afull[s], ph);
        if (wu.kb < wu.ke && !ready) ok = false;
        bool done0 = false;
        for (int k = wu.kb; ok && k < wu.ke; ++k, ++it) {
          tc_fence_after();
          const uint64_t ad = ad0 + uint64_t(s * (L::A_BYTES >> 4));
          const uint64_t bd = bd0 + uint64_t(s * (L::X_BYTES >> 4));
          const uint32_t s1 = (s + 1 == uint32_t(NS)) ? 0u : s + 1;
          const uint32_t ph1 = (s + 1 == uint32_t(NS)) ? (ph ^ 1u) : ph;
          bool next_ready = false;
#pragma unroll
          for (int kk = 0; kk < G_K / 16; ++kk) {
            // K-major 128B swizzle: advance 32 B per 16 K; MN-major: two 8-row atoms (2 KB).
            const uint64_t a_kk = ad + uint64_t(kk * (BWD ? 2048 / 16 : 32 / 16));
            const uint64_t b_kk = bd + uint64_t(kk * (32 / 16));
            mma(d0, a_kk, b_kk, id0, acc0 || kk > 0);
            if (kk == 0 && k + 1 < wu.ke) next_ready = mbar_test_wait(&afull[s1], ph1);
          }
          acc0 = true;
          if (PAIR && k + 1 == wu.ke) {
            commit_both(&acc_full[0]);
            done0 = true;
          }
          if (PAIR && n1 > 0) {
            if (!take1()) {
              ok = false;
              ++it;
              break;
            }
            tc_fence_after();
            // the same decoded weight stage against the stage's second token half (16 KB on)
#pragma unroll
            for (int kk = 0; kk < G_K / 16; ++kk) {
              const uint64_t a_kk = ad + uint64_t(kk * (BWD ? 2048 / 16 : 32 / 16));
              const uint64_t b_kk = bd + uint64_t((L::X_BYTES / 2) >> 4) + uint64_t(kk * (32 / 16));
              mma(d1, a_kk, b_kk, id1, acc1 || kk > 0);
            }
            acc1 = true;
          }
          commit_both(&empty[s]);
          s = s1;
          ph = ph1;
          if (k + 1 < wu.ke && !next_ready && !pwait(&afull[s], ph)) {
            ok = false;
            ++it;
            break;
          }
        }
        if (!done0) commit_both(&acc_full[b]);
        if (PAIR) {
          if (!take1()) ok = false;
          commit_both(&acc_full[1]);
        }
      }
      // every MMA must be complete before TMEM is released
      commit_both(mma_done);
      drain_wait(mma_done, 0);
    } else if (PAIR && lane == 0) {
      drain_wait(mma_done, 0);
    }
  } else {
   const bool epi = warp >= G_EPI_WARP0;
   if (!epi || g.epi_decode) {
    // ------------------------------------------------------------ decode warps
    // Two groups of four warps (below); group g decodes the stages whose global index
    // is g modulo the group count (so every ring slot has one owner), each thread one whole
    // 64-value block row per stage: one scale and one 16-entry table per 64 values.  In a
    // backward launch where every CTA has at most one work unit (`epi_decode`), the epilogue
    // warps have nothing to do until that unit's accumulator is ready, so they decode as groups
    // 2 and 3 first: each group then has four stage-times for its stage,
    // which hides the lag of the decode warp that shares the MMA issuer's SM sub-partition.
    //  forward : row d of the K-major tile = weight row m0 + d, K columns 64 kl .. +63 of the
    //            stage; packed row d of the stage is 32 B in the 32B swizzle (16-byte chunk c
    //            at c ^ ((d >> 2) & 1)), so a warp's 16-byte loads hit all 32 banks.
    //  backward: K row r = d & 63 of the MN-major tile = weight row 64 kl + r, tile columns
    //            64 j .. +63 with j = d >> 6 (one 128-byte row of M chunk j); packed row r has
    //            64 B in the 64B swizzle (16-byte chunk c at c ^ ((r >> 1) & 3)), the thread's
    //            two chunks are 2j and 2j + 1.
    // Each group takes the two oldest and the two youngest warps of its role (decode: warps
    // 2, 3, 8, 9 and 4-7; epilogue: 10, 11, 16, 17 and 12-15), one on every SM sub-partition
    // either way.  A sub-partition's scheduler favours its older warps, so with warps 2-5 and
    // 6-9 one group decoded every stage behind the other.
    const int wrel = warp - (epi ? G_EPI_WARP0 : G_DQ_WARP0);  // 0..7
    const int dq = (((((wrel + 2) >> 2) & 1) << 2) + ((wrel + 2) & 3)) * 32 + lane;  // 0..255
    const int ngrp = g.epi_decode ? 4 : 2;
    const int grp = (dq >> 7) + (epi ? 2 : 0);
    const int d = dq & 127;
    float code[16];  // NF4 code of the current weight (reloaded when the weight changes)
    int code_seg = -1;
    const int r = BWD ? (d & 63) : d;
    const int j = BWD ? (d >> 6) : 0;
    const int sw = (r >> 1) & 3;
    const uint32_t sw32 = uint32_t((r >> 2) & 1);
    const uint32_t p_off0 = BWD ? uint32_t(r * 64 + (((2 * j) ^ sw) << 4)) : uint32_t(r * 32) + (sw32 << 4);
    const uint32_t p_off1 = BWD ? uint32_t(r * 64 + (((2 * j + 1) ^ sw) << 4))
                                : uint32_t(r * 32) + ((1u ^ sw32) << 4);
    // GLU: packed row d is row d & 63 of gate (d < 64) or of up; it goes to operand row
    // 32 q + 16 (up) + i for feature 16 q + i, so TMEM lanes i and i + 16 of an epilogue warp
    // hold the gate and up rows of one feature
    const int rrow = GLUF ? (d & 63) : r;  // row of its weight, from the tile's m0
    const int arow = GLUF ? 32 * ((d & 63) >> 4) + 16 * (d >> 6) + (d & 15) : r;
    const uint32_t a_off = uint32_t(j * 8192 + (arow >> 3) * 1024 + (arow & 7) * 128);
    const uint32_t key = uint32_t(arow & 7);
    const uint32_t k16 = g.k16, k31 = g.k16 << 15;

    uint32_t it = 0, lc = 0;
    bool ok = true;
    for (int u = unit0; ok && u < nunits; u += ustride) {
      const WorkUnit wu = u == unit0 ? wu_first : work_unit<MULTI, PAIR, GLUF>(g, u, rank);
      const TileCoord& tc = wu.tc;
      // the tile's weight (forward; GLU: this thread's row's); weight 0 backward
      const int tws = GLUF ? (d >> 6) : (MULTI ? tc.seg : 0);
      const GemmW& W = g.w[tws];
      // one slab per adapter (a K-concatenated backward may carry several), in the order the
      // MMA issuer consumes them
      for (int li = 0; !epi && wu.split == 0 && li < (KCAT ? g.nw : 1); ++li) {
        const GemmW& WL = KCAT ? g.w[li] : W;
        if (!WL.has_lora) continue;
        if (!pwait(lora_empty, (lc & 1) ^ 1)) {
          ok = false;
          break;
        }
        ++lc;
        const uint32_t la = sbase + L::LA;
        const uint32_t lb = sbase + L::LB;
        if (dq < G_M) {
          if (!BWD) {
            const int64_t o = tc.m0 + dq;  // s * B[o, 0:16]
            uint4 v0 = make_uint4(0, 0, 0, 0), v1 = v0;
            if (o < WL.out_f) {
              const uint4* src = reinterpret_cast<const uint4*>(WL.lora_w + o * 16);
              v0 = scale_pack8(__ldg(src), WL.lora_scale);
              v1 = scale_pack8(__ldg(src + 1), WL.lora_scale);
            }
            st_shared_v4(la + slab_off(dq, 0), v0);
            st_shared_v4(la + slab_off(dq, 1), v1);
          } else {
            const int64_t i = tc.m0 + dq;  // s * A[0:16, i]
            float v[16];
#pragma unroll
            for (int rr = 0; rr < 16; ++rr)
              v[rr] = (i < g.in_f) ? __half2float(WL.lora_w[int64_t(rr) * g.in_f + i]) * WL.lora_scale
                                   : 0.f;
            st_shared_v4(la + slab_off(dq, 0),
                         make_uint4(pack_half2(v[0], v[1]), pack_half2(v[2], v[3]),
                                    pack_half2(v[4], v[5]), pack_half2(v[6], v[7])));
            st_shared_v4(la + slab_off(dq, 1),
                         make_uint4(pack_half2(v[8], v[9]), pack_half2(v[10], v[11]),
                                    pack_half2(v[12], v[13]), pack_half2(v[14], v[15])));
          }
        }
        // token side: X_ROWS rows x 2 chunks of 16 B.  A pair: slab row t is row t & 127 of
        // MMA half h = t >> 7 in this CTA, i.e. token 256 h + rank n_h / 2 + (t & 127) of the
        // tile, present when t & 127 < n_h / 2.
#pragma unroll
        for (int jj = 0; jj < L::X_ROWS / 128; ++jj) {
          const int c = dq + 256 * jj;
          const int t = c >> 1, kc = c & 1;
          int tok = t;
          bool in = true;
          if (PAIR) {
            const int h = t >> 7, tl = t & 127;
            const int nhalf = min(tc.tn - h * G_NMAX, G_NMAX) / 2;
            tok = h * G_NMAX + int(rank) * nhalf + tl;
            in = tl < nhalf;
          }
          uint4 v = make_uint4(0, 0, 0, 0);
          if (in && tok < tc.tn_real)
            v = __ldg(reinterpret_cast<const uint4*>(WL.lora_t + (tc.t0 + tok) * 16 + kc * 8));
          st_shared_v4(lb + slab_off(t, kc), v);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) arrive_issuer(lora_full, lora_full_l);
      }
      if (!ok) break;

      const int64_t col = BWD ? (tc.m0 + 64 * j) : 0;
      const bool lane_valid = BWD ? (col < g.in_f) : (tc.m0 + rrow < W.out_f);
      // weight of stage k, and the element offset of the thread's first value in it
      struct Src {
        ScaleSrc v;
        int ws;
      };
      auto src = [&](int k) -> Src {
        Src x{ScaleSrc{0u, 0.f}, KCAT ? 0 : tws};
        if (k >= wu.ke) return x;
        if (KCAT) x.ws = kseg(g, k);
        const GemmW& Wk = g.w[KCAT ? x.ws : tws];
        const int kl = KCAT ? k - kbeg(g, x.ws) : k;
        const int64_t e = BWD ? int64_t(kl * G_K + r) * g.in_f + col : (tc.m0 + rrow) * g.in_f + int64_t(kl) * G_K;
        x.v = load_scale_src(Wk, e >> Wk.log2_bs, lane_valid);
        return x;
      };
      const float off_t = W.nested ? __ldg(W.offset) : 0.f;  // the tile's weight
      auto scale_of = [&](const Src& x) -> float {
        if (!lane_valid) return 0.f;
        const GemmW& Wk = g.w[KCAT ? x.ws : tws];
        const int sg = KCAT ? x.ws : tws;
        const float off = KCAT ? (Wk.nested ? __ldg(Wk.offset) : 0.f) : off_t;
        return Wk.nested ? __fadd_rn(__fmul_rn(s_code2[256 * sg + x.v.q], x.v.a), off) : x.v.a;
      };
      // blocksize 32: the second 32 values of a row are their own block
      auto second_half_scale = [&](int k) -> float {
        Src x{ScaleSrc{0u, 0.f}, KCAT ? kseg(g, k) : tws};
        const GemmW& Wk = g.w[x.ws];
        const int kl = KCAT ? k - kbeg(g, x.ws) : k;
        const int64_t e = BWD ? int64_t(kl * G_K + r) * g.in_f + col + 32
                              : (tc.m0 + rrow) * g.in_f + int64_t(kl) * G_K + 32;
        x.v = load_scale_src(Wk, e >> Wk.log2_bs, lane_valid);
        return scale_of(x);
      };
      // this group's stages of the unit: k0, k0 + ngrp, ...; scales of the next two in flight
      const int k0 = wu.kb + int((uint32_t(grp) - it) & uint32_t(ngrp - 1));
      float sc = scale_of(src(k0));
      Src raw1 = src(k0 + ngrp);
      for (int k = k0; k < wu.ke; k += ngrp) {
        const int ws = KCAT ? kseg(g, k) : tws;
        if (ws != code_seg) {
          code_seg = ws;
#pragma unroll
          for (int i = 0; i < 16; ++i) code[i] = s_code[16 * ws + i];
        }
        const uint32_t its = it + uint32_t(k - wu.kb);
        const int s = its % NS;
        const uint32_t ph = (its / NS) & 1;
        const Nf4Table tab = make_table(code, sc);
        const Src raw2 = src(k + 2 * ngrp);
        const float sc1 = scale_of(raw1);
        if (!pwait(&full[s], ph)) {
          ok = false;
          break;
        }
        const uint4 w0 = ld_shared_v4(sbase + L::P + s * L::P_BYTES + p_off0);
        const uint4 w1 = ld_shared_v4(sbase + L::P + s * L::P_BYTES + p_off1);
        const uint32_t abase = sbase + L::A + s * L::A_BYTES + a_off;
        const uint32_t wa[4] = {w0.x, w0.y, w0.z, w0.w};
#pragma unroll
        for (int c = 0; c < 4; ++c)
          st_shared_v4(abase + ((uint32_t(c) ^ key) << 4), decode_word_f16_mh(tab, wa[c], k16, k31));
        const uint32_t wb[4] = {w1.x, w1.y, w1.z, w1.w};
        if (g.w[ws].log2_bs == 5) {
          const Nf4Table tab2 = make_table(code, second_half_scale(k));
#pragma unroll
          for (int c = 0; c < 4; ++c)
            st_shared_v4(abase + ((uint32_t(4 + c) ^ key) << 4), decode_word_f16_mh(tab2, wb[c], k16, k31));
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c)
            st_shared_v4(abase + ((uint32_t(4 + c) ^ key) << 4), decode_word_f16_mh(tab, wb[c], k16, k31));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) arrive_issuer(&afull[s], afull_l + 8u * uint32_t(s));
        sc = sc1;
        raw1 = raw2;
      }
      it += uint32_t(wu.ke - wu.kb);
    }
   }
   if (epi) {
    // --------------------------------------------------------------- epilogue
    // Warp w may only read TMEM lanes 32*(w%4)..+31 (the tile's weight rows); the two
    // groups of four warps take alternate 32-column chunks.  Lanes 2i and 2i+1 hold
    // adjacent weight rows, i.e. adjacent output columns: each lane packs its two tokens
    // j, j+1 into a half2, swaps it with its neighbour, and one byte permute gives the even
    // lane (row, row+1) of token j and the odd lane the same two columns of token j+1.
    const int lq = warp & 3;
    const int grp = (warp - G_EPI_WARP0) >> 2;
    const bool odd = (lane & 1) != 0;
    const uint32_t xsel = odd ? 0x3276u : 0x5410u;
    constexpr bool split = SPLIT;
    const int nparts = SPLIT ? g.splits - 1 : 0;
    const bool leader = threadIdx.x == 32 * G_EPI_WARP0;
    volatile int* s_ticket = reinterpret_cast<volatile int*>(smem + L::MISC + 8);  // [2]
    uint32_t lt = 0;
    for (int u = unit0; u < nunits; u += ustride, ++lt) {
      const WorkUnit wu = u == unit0 ? wu_first : work_unit<MULTI, PAIR, GLUF>(g, u, rank);
      // split-K bookkeeping is per CTA: a pair's two 128-row halves are separate tiles there
      const int ctile = PAIR ? 2 * wu.tile + int(rank) : wu.tile;
      const TileCoord& tc = wu.tc;
      // GLU: lanes 0-15 of a warp hold gate rows, lanes 16-31 the up rows of the same features
      const int glu_up = GLUF ? (lane >> 4) : 0;
      const GemmW& W = g.w[GLUF ? glu_up : (MULTI ? tc.seg : 0)];
      const int64_t ld_out = BWD ? g.in_f : W.out_f;
      // single CTAs: accumulator b of two; a pair: the tile's 512 columns, handed over in two
      // halves (acc_full[0] / [1]); split-K takes both halves at once
      const uint32_t b = PAIR ? 0u : (lt & 1);
      const uint32_t fpar = PAIR ? (lt & 1) : ((lt >> 1) & 1);
      constexpr bool by_half = PAIR && !SPLIT;
      // uniform over the warp (tcgen05.ld is warp-collective) and, for split-K, over all
      // epilogue warps (they meet at named barriers below)
      bool ok = pwait(&acc_full[b], fpar);
      if (PAIR && SPLIT) ok = ok && pwait(&acc_full[1], fpar);
      ok = split ? epi_bar_and(ok) : __all_sync(0xffffffffu, ok);
      tc_fence_after();
      if (!ok) break;
      const int prow = 32 * lq + lane;  // accumulator row = TMEM lane
      // output column of this lane's row (GLU: the feature; lanes 2i, 2i+1 stay adjacent)
      const int64_t row = GLUF ? tc.m0 + 16 * lq + (lane & 15) : tc.m0 + prow;
      const bool row_ok = row < ld_out;  // ld_out is a multiple of 64: pairs are all in or out
      const uint32_t taddr = tmem_base + (uint32_t(32 * lq) << 16) + b * G_ACC_COLS;
      constexpr int ACC_T = acc_tokens<PAIR>();
      bool fail = false;
      // Split-K: every K range of a tile takes a ticket; all but the last write their fp32
      // partial to the workspace slot of their range, the last sums the ranges in range
      // order (its own from TMEM) and writes the output, so the result does not depend on
      // which range finishes last.  The last one only waits for ranges that already hold
      // tickets, i.e. are past their main loops, so the wait cannot depend on unscheduled work.
      int ticket = nparts;
      if (split) {
        // the test hook's unit behaves as a range that gave up before its ticket: it takes
        // none and writes nothing, so no range of its tile sums the partials
        if (leader) s_ticket[lt & 1] = u == g.drop_ticket_unit ? -1 : atomicAdd(g.ws_cnt + ctile, 1);
        epi_bar_sync();
        ticket = s_ticket[lt & 1];
      }
      // partial tiles are column-major [tokens][128 rows]: for one token the 32 lanes of a
      // warp (32 consecutive rows) touch one 128-byte line
      const float* tile_part = g.ws_part + int64_t(ctile) * (nparts + 1) * (G_M * ACC_T);
      const float* part0 = tile_part + prow;
      // The last range of a tile on its CTA's last unit reads the other ranges' partials
      // through bulk copies into the ring, which that unit's completed accumulator leaves idle
      // (every stage it loaded or decoded has been consumed by its MMAs): rounds of 64 tokens,
      // two rounds in flight, each round one 32 KB slice [64 tokens][128 rows] per range.
      // Per-thread L2 loads of the same slices are bound by their latency (the bytes one
      // thread can keep in flight); the bulk copies are not.
      const bool staged = SPLIT && g.red_staged != 0 && ticket == nparts && nparts >= 1 &&
                          nparts <= L::RED_PARTS && u + ustride >= nunits;
      const int nrounds = staged ? (tc.tn + 63) >> 6 : 0;
      int red_issued = 0;  // rounds the leader has issued
      auto issue_round = [&](int r) {
        ++red_issued;
        const int bsl = r & 1;
        mbar_arrive_expect_tx(&red_full[bsl], uint32_t(nparts) * uint32_t(L::RED_SLICE));
        int j = 0;
        for (int sp = 0; sp <= nparts; ++sp) {
          if (sp == wu.split) continue;
          bulk_load_g2s(sbase + uint32_t((L::RED_PARTS * bsl + j) * L::RED_SLICE),
                        tile_part + int64_t(sp) * (G_M * ACC_T) + int64_t(64 * r) * G_M,
                        uint32_t(L::RED_SLICE), smem_u32(&red_full[bsl]));
          ++j;
        }
      };
      if (ticket < 0) {
        if (leader) atomicExch(&g_gemm_error, 4);
      } else if (ticket < nparts) {
        float* dst = const_cast<float*>(part0) + int64_t(wu.split) * (G_M * ACC_T);
        for (int c0 = 32 * grp; c0 < tc.tn; c0 += 64) {
          uint32_t acc[32];
          tmem_ld_32x32b_x32(taddr + uint32_t(c0), acc);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) __stcg(dst + (c0 + j) * G_M, __uint_as_float(acc[j]));
        }
        __threadfence();
        epi_bar_sync();
        if (leader) atomicAdd(g.ws_cnt + G_SPLIT_MAX_TILES + ctile, 1);
      } else {
        if (split) {
          if (leader) {
            const bool arrived = wait_count(g.ws_cnt + G_SPLIT_MAX_TILES + ctile, nparts);
            if (!arrived) *abort_flag = 1;
            g.ws_cnt[ctile] = 0;  // every range of the tile has arrived: reset for reuse
            g.ws_cnt[G_SPLIT_MAX_TILES + ctile] = 0;
            __threadfence();
            if (staged && arrived) {
              // the partials were published by other CTAs' generic stores and the count's
              // acquire; the bulk copies read them through the async proxy
              fence_proxy_async_global();
              issue_round(0);
              if (nrounds > 1) issue_round(1);
            }
          }
          epi_bar_sync();
        }
        const bool has_bias = !BWD && W.bias != nullptr;
        const float bias_v = (has_bias && row_ok) ? __half2float(W.bias[row]) : 0.f;
        // this lane's first token of a chunk is c0 + odd; it stores every other token
        uint32_t* outp = reinterpret_cast<uint32_t*>(W.out + (tc.t0 + (odd ? 1 : 0)) * ld_out +
                                                     (row & ~int64_t(1)));
        // 16 half2 stores of one 32-token chunk; lim: the lane's stores with jj < lim land
        // SwiGLU epilogue of one 32-token chunk: this lane's gate or up row to its output (as
        // emit), then m = fp16(g * sigmoid(g) * u) from the fp16 g and u -- each lane trades
        // half of its chunk with lane ^ 16, so lanes 0-15 get tokens 0-15 of their feature and
        // lanes 16-31 tokens 16-31 -- stored with the same neighbour pairing
        uint32_t* moutp = GLUF ? reinterpret_cast<uint32_t*>(g.glu_out + (tc.t0 + (odd ? 1 : 0)) * ld_out +
                                                             (row & ~int64_t(1)))
                               : nullptr;
        auto glu_emit = [&](const uint32_t (&acc)[32], int c0) {
          uint32_t hp[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) hp[k] = pack_half2(__uint_as_float(acc[2 * k]), __uint_as_float(acc[2 * k + 1]));
          const int lim = row_ok ? tc.tn_real - c0 - (odd ? 1 : 0) : 0;
          uint32_t* p = outp + ((int64_t(c0) * ld_out) >> 1);
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const uint32_t h = prmt(hp[k], __shfl_xor_sync(0xffffffffu, hp[k], 1), xsel);
            if (2 * k < lim) p[int64_t(k) * ld_out] = h;
          }
          uint32_t mp[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t other = __shfl_xor_sync(0xffffffffu, glu_up ? hp[k] : hp[8 + k], 16);
            const uint32_t gg = glu_up ? other : hp[k];
            const uint32_t uu = glu_up ? hp[8 + k] : other;
            const float2 gf = __half22float2(*reinterpret_cast<const __half2*>(&gg));
            const float2 uf = __half22float2(*reinterpret_cast<const __half2*>(&uu));
            mp[k] = pack_half2(gf.x * glu_sigmoid(gf.x) * uf.x, gf.y * glu_sigmoid(gf.y) * uf.y);
          }
          const int base = glu_up ? 16 : 0;
          const int limm = row_ok ? tc.tn_real - c0 - base - (odd ? 1 : 0) : 0;
          uint32_t* pm = moutp + ((int64_t(c0 + base) * ld_out) >> 1);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t h = prmt(mp[k], __shfl_xor_sync(0xffffffffu, mp[k], 1), xsel);
            if (2 * k < limm) pm[int64_t(k) * ld_out] = h;
          }
        };
        // SwiGLU backward epilogue of one 32-token chunk (dX of down = dm): for the lane's word
        // (row, row + 1) at token c0 + jj + odd -- the word the dm store would write -- read the
        // forward's gate and up words at the same place and write
        //   dup = fp16(dm * g * sig), dgate = fp16(dm * u * sig * (1 + g * (1 - sig)))
        // with dm rounded to fp16 first (nf4b_swiglu_bwd's arithmetic, bit for bit); all 32
        // gate and up words of the chunk are loaded before any is used (one DRAM round trip per
        // chunk: the drain is bound by the loads' latency)
        auto glub_emit = [&](const uint32_t (&acc)[32], int c0) {
          const int lim = row_ok ? tc.tn_real - c0 - (odd ? 1 : 0) : 0;
          const int64_t w0 = ((tc.t0 + c0 + (odd ? 1 : 0)) * ld_out + (row & ~int64_t(1))) >> 1;
          const uint32_t* gw = reinterpret_cast<const uint32_t*>(g.glu_g) + w0;
          const uint32_t* uw = reinterpret_cast<const uint32_t*>(g.glu_u) + w0;
          uint32_t* dgw = reinterpret_cast<uint32_t*>(g.glu_dg) + w0;
          uint32_t* duw = reinterpret_cast<uint32_t*>(g.glu_du) + w0;
          uint32_t gv[16], uv[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const int jj = 2 * q;
            const int64_t o = int64_t(q) * ld_out;
            gv[q] = jj < lim ? __ldcs(gw + o) : 0u;
            uv[q] = jj < lim ? __ldcs(uw + o) : 0u;
          }
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t dmw[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const int jj = 16 * hh + 2 * q;
              const uint32_t own = pack_half2(__uint_as_float(acc[jj]), __uint_as_float(acc[jj + 1]));
              dmw[q] = prmt(own, __shfl_xor_sync(0xffffffffu, own, 1), xsel);
            }
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const int jj = 16 * hh + 2 * q;
              const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&dmw[q]));
              const float2 gg = __half22float2(*reinterpret_cast<const __half2*>(&gv[8 * hh + q]));
              const float2 uu = __half22float2(*reinterpret_cast<const __half2*>(&uv[8 * hh + q]));
              const float s0 = glu_sigmoid(gg.x), s1 = glu_sigmoid(gg.y);
              const uint32_t du = pack_half2(dm.x * gg.x * s0, dm.y * gg.y * s1);
              const uint32_t dg = pack_half2(dm.x * uu.x * s0 * (1.f + gg.x * (1.f - s0)),
                                             dm.y * uu.y * s1 * (1.f + gg.y * (1.f - s1)));
              if (jj < lim) {
                const int64_t o = int64_t(jj >> 1) * ld_out;
                duw[o] = du;
                dgw[o] = dg;
              }
            }
          }
        };
        auto emit = [&](const uint32_t (&acc)[32], int c0, auto bias_c, int lim) {
          uint32_t* p = outp + ((int64_t(c0) * ld_out) >> 1);
#pragma unroll
          for (int jj = 0; jj < 32; jj += 2) {
            float v0 = __uint_as_float(acc[jj]), v1 = __uint_as_float(acc[jj + 1]);
            if (decltype(bias_c)::value) {
              v0 += bias_v;
              v1 += bias_v;
            }
            const uint32_t own = pack_half2(v0, v1);  // tokens c0+jj, c0+jj+1 of this row
            const uint32_t h = prmt(own, __shfl_xor_sync(0xffffffffu, own, 1), xsel);
            if (jj < lim) p[int64_t(jj >> 1) * ld_out] = h;
          }
        };
        for (int h = 0; h < (by_half ? 2 : 1); ++h) {
          const int cb = by_half ? h * G_NMAX : 0;
          const int ce = (by_half && h == 0) ? min(tc.tn, G_NMAX) : tc.tn;
          if (by_half && h == 1) {
            // half 0 drained: hand it back to the MMA issuer, then take half 1
            tc_fence_before();
            __syncwarp();
            if (lane == 0) arrive_issuer(&acc_empty[0], acc_empty_l);
            const bool ok1 = __all_sync(0xffffffffu, pwait(&acc_full[1], fpar));
            tc_fence_after();
            if (!ok1) {
              fail = true;
              break;
            }
          }
          // staged: every epilogue thread takes every round (they meet at a named barrier per
          // round), a group whose chunk c0 lies past the tile only waits
          for (int c0 = cb + 32 * grp, r = 0; staged ? r < nrounds : c0 < ce; c0 += 64, ++r) {
            if (staged) {
              // every thread is past round r - 1, whose buffer the leader refills with round r + 1
              // (generic reads of it ordered before those async-proxy writes)
              if (r > 0) fence_proxy_async_smem();
              const bool okr = epi_bar_and(pwait(&red_full[r & 1], uint32_t(r >> 1) & 1u));
              if (!okr) {
                // no bulk copy may still be landing in the ring at exit
                if (leader)
                  for (int rr = r; rr < red_issued; ++rr) drain_wait(&red_full[rr & 1], uint32_t(rr >> 1) & 1u);
                fail = true;
                break;
              }
              if (leader && r >= 1 && r + 1 < nrounds) issue_round(r + 1);
              if (c0 >= ce) continue;
            }
            uint32_t acc[32];
            if (!SPLIT) {
              tmem_ld_32x32b_x32(taddr + uint32_t(c0), acc);
              tmem_ld_wait();
            } else {
              // the 32 columns summed in range order, one range per round (this CTA's own
              // range from TMEM): the reduction is bound by L2 round trips, so each round has
              // all 32 loads of a thread in flight
#pragma unroll
              for (int j = 0; j < 32; ++j) acc[j] = __float_as_uint(0.f);
              for (int sp = 0; sp <= nparts; ++sp) {
                uint32_t v[32];
                if (sp == wu.split) {
                  tmem_ld_32x32b_x32(taddr + uint32_t(c0), v);
                  tmem_ld_wait();
                } else if (staged) {
                  const float* src = reinterpret_cast<const float*>(
                                         smem + (L::RED_PARTS * (r & 1) + sp - (sp > wu.split ? 1 : 0)) * L::RED_SLICE) +
                                     (c0 - 64 * r) * G_M + prow;
#pragma unroll
                  for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(src[j * G_M]);
                } else {
                  const float* src = part0 + int64_t(sp) * (G_M * ACC_T) + c0 * G_M;
#pragma unroll
                  for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__ldcg(src + j * G_M));
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) acc[j] = __float_as_uint(__uint_as_float(acc[j]) + __uint_as_float(v[j]));
              }
            }
            // stores of token c0 + jj + odd land while that token is in the tile; the paths
            // below are warp-uniform (emit shuffles across the warp)
            if (GLUF) {
              glu_emit(acc, c0);
              continue;
            }
            if (GLU && BWD) {
              glub_emit(acc, c0);
              continue;
            }
            const int lim = row_ok ? tc.tn_real - c0 - (odd ? 1 : 0) : 0;
            const bool whole = __all_sync(0xffffffffu, lim >= 32);
            if (has_bias) {
              if (whole)
                emit(acc, c0, std::true_type(), 32);
              else
                emit(acc, c0, std::true_type(), lim);
            } else {
              if (whole)
                emit(acc, c0, std::false_type(), 32);
              else
                emit(acc, c0, std::false_type(), lim);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (!PAIR) {
          arrive_issuer(&acc_empty[b], acc_empty_l + 8u * b);
        } else {
          if (SPLIT) arrive_issuer(&acc_empty[0], acc_empty_l);
          if (!fail) arrive_issuer(&acc_empty[1], acc_empty_l + 8u);
        }
      }
      if (fail) break;
    }
   }
  }

  tc_fence_before();
  __syncthreads();
  if (SPLIT && threadIdx.x == 0) {
    // the last CTA to get here clears the counters of every tile of the launch (the last
    // range of a tile has normally done so already; a range that gave up may have left its
    // tile's counts behind) and the exit count itself
    __threadfence();
    if (atomicAdd(g.ws_cnt + G_SPLIT_EXIT, 1) == int(gridDim.x) - 1) {
      const int ctiles = g.m_tiles * g.n_tiles * (PAIR ? 2 : 1);
      for (int i = 0; i < ctiles; ++i) {
        g.ws_cnt[i] = 0;
        g.ws_cnt[G_SPLIT_MAX_TILES + i] = 0;
      }
      g.ws_cnt[G_SPLIT_EXIT] = 0;
      __threadfence();
    }
  }
  // a pair: neither CTA leaves (or frees TMEM) while the other may still touch its shared
  // memory or barriers
  if (PAIR) cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem_base, G_TMEM_COLS);
    else
      tmem_dealloc(tmem_base, G_TMEM_COLS);
  }
}

// ------------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

static int make_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner,
                        uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                        CUtensorMapSwizzle sw) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    record_driver_error("cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)", -1);
    return NF4B_ERR_CUDA;
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    record_driver_error("cuTensorMapEncodeTiled", int(r));
    return NF4B_ERR_CUDA;
  }
  return NF4B_OK;
}

static int sm_count_cached() {
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

template <bool BWD, bool SPLIT, bool MULTI, bool PAIR, bool GLU = false>
static int set_smem_attr() {
  static std::mutex mu;
  static bool done[64] = {false};
  int dev = 0;
  NF4B_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return NF4B_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(mu);
  if (!done[dev]) {
    NF4B_CUDA_TRY(cudaFuncSetAttribute(nf4_gemm_kernel<BWD, SPLIT, MULTI, PAIR, GLU>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, Smem<PAIR>::ALLOC));
    done[dev] = true;
  }
  return NF4B_OK;
}

// Launch configuration of a 2-CTA cluster launch of `grid` CTAs (programmatic launch as for
// single CTAs, unless `pdl` is false).
struct PairLaunch {
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[2];
  PairLaunch(unsigned grid, cudaStream_t s, bool pdl) : cfg{}, attr{} {
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(G_THREADS, 1, 1);
    cfg.dynamicSmemBytes = Smem<true>::ALLOC;
    cfg.stream = s;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
  }
};

// CTA pairs (2-CTA clusters, one CTA per SM) that can be resident at once; 0 when the
// device cannot run them.
static int pair_slots_cached() {
  static std::mutex mu;
  static int cached[64] = {0};  // 0: not asked yet; -1: unavailable
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == 0) {
    int n = 0;
    if (set_smem_attr<false, false, false, true>() == NF4B_OK) {
      PairLaunch pl(2u * unsigned(sm_count_cached()), nullptr, false);
      if (cudaOccupancyMaxActiveClusters(&n, nf4_gemm_kernel<false, false, false, true, false>, &pl.cfg) !=
          cudaSuccess)
        n = 0;
    }
    cudaGetLastError();  // a refused query leaves no sticky error behind
    cached[dev] = n > 0 ? n : -1;
  }
  return cached[dev] > 0 ? cached[dev] : 0;
}

// Tiling of one launch.  Single CTAs: 128-row weight tiles x 256-token (or 128-token) tiles
// on one CTA per SM.  Pairs: 256-row x 512-token tiles (each weight's rows rounded up to 256)
// on 2-CTA clusters.  The
// K stages of a tile may be split into `splits` ranges when there are fewer tiles than slots.
struct GemmPlan {
  int64_t m_tiles, n_tiles, tiles;
  int32_t nk;
  int32_t splits;
  int32_t tile_n;  // tokens per tile
  bool pair;
  int64_t slots;  // CTAs (single) or clusters (pair) resident at once
};

constexpr int G_MAX_SPLITS = 8;

// Cost model in stage-times of a 256-token tile (~0.7 us) of the busiest slot: a unit costs its
// stages plus ~3 of pipeline fill and drain; a split tile adds the round trip of its fp32
// partials through L2, measured at ~3 us to write one 128 x 256 partial and ~3 us per partial
// for the last CTA to read back (4 + 4 per partial).  A 128-token tile's stage costs ~0.55 of
// a 256-token one (the decode of the weight stage is the same, the MMA half) and its partials
// half as much.  A pair's 512-token tile (two MMAs per decoded stage, on two SMs) runs a stage
// in ~1.35 and adds ~8 per tile (its single accumulator leaves the 512-column drain exposed);
// its CTAs' partials are twice as large.  (Fitted to CUDA-event times of the seven
// Qwen2.5-1.5B projection shapes, forward and backward, at 1170, 2048 and 8192 tokens.)
static double plan_cost(int64_t tiles, int64_t slots, int32_t nk, int64_t sp, int32_t tile_n) {
  const double stage = tile_n == 128 ? 0.55 : (tile_n == 256 ? 1.0 : 1.35);
  const double fill = tile_n == G_PAIR_TILE_N ? 8.0 : 3.0;
  const double red = double(tile_n) / 64.0;
  const int64_t waves = (tiles * sp + slots - 1) / slots;
  const double reduce = sp > 1 ? red * double(sp) : 0.0;
  return double(waves) * (stage * double((nk + sp - 1) / sp) + fill) + reduce;
}

// Split-K choice: a split must beat the unsplit launch by 5 % and leave every range at least 2
// stages.  Returns the plan's cost.
static double plan_splits(GemmPlan* p, int64_t max_tiles) {
  p->splits = 1;
  double best = plan_cost(p->tiles, p->slots, p->nk, 1, p->tile_n);
  if (p->tiles <= 0 || p->tiles >= p->slots || p->tiles > max_tiles) return best;
  for (int sp = 2; sp <= G_MAX_SPLITS && p->nk / sp >= 2; ++sp) {
    const double c = plan_cost(p->tiles, p->slots, p->nk, sp, p->tile_n);
    if (c < 0.95 * best) {
      best = c;
      p->splits = sp;
    }
  }
  return best;
}

// Token tile width from STEW_NF4_TILE_N: "128" or "256" forces it (single CTAs), otherwise the
// cost model chooses.
static int tile_n_env() {
  const char* v = std::getenv("STEW_NF4_TILE_N");
  if (v == nullptr || v[0] == '\0') return 0;
  return std::atoi(v) == 128 ? 128 : 256;
}

// K ranges per tile from STEW_NF4_SPLITS ("1" to "8"; 0 = the cost model's choice): applied to
// the chosen tiling when it may split (fewer tiles than the workspace's counters, at least two
// stages a range).
static int splits_env() {
  const char* v = std::getenv("STEW_NF4_SPLITS");
  if (v == nullptr || v[0] == '\0') return 0;
  const int k = std::atoi(v);
  return (k >= 1 && k <= G_MAX_SPLITS) ? k : 0;
}

// Pair mode from STEW_NF4_PAIR: "0" never, "1" whenever the device runs pairs, otherwise
// automatic.
static int pair_mode_env() {
  const char* v = std::getenv("STEW_NF4_PAIR");
  if (v == nullptr || v[0] == '\0') return -1;
  return v[0] == '0' ? 0 : 1;
}

// Split-K reduction through bulk copies into the idle ring (STEW_NF4_SPLIT_STAGED: "0" reads
// the partials with per-thread L2 loads instead; both sum in the same order, bit for bit).
static int red_staged_env() {
  const char* v = std::getenv("STEW_NF4_SPLIT_STAGED");
  return (v != nullptr && v[0] == '0') ? 0 : 1;
}

static GemmPlan force_splits(GemmPlan p) {
  const int k = splits_env();
  const int64_t max_tiles = p.pair ? G_SPLIT_MAX_TILES / 2 : G_SPLIT_MAX_TILES;
  if (k > 0 && p.tiles > 0 && p.tiles <= max_tiles && p.nk / k >= 2) p.splits = k;
  return p;
}

// rows: the M-side rows of each weight of the launch (forward: out features of each grouped
// weight; backward: the in features, once).  kdim: the reduction length.
static GemmPlan plan_gemm(int64_t n, const int64_t* rows, int nrows, int64_t kdim) {
  GemmPlan single{};
  single.tile_n = G_NMAX;
  single.n_tiles = (n + G_NMAX - 1) / G_NMAX;
  single.nk = int32_t(kdim / G_K);
  single.pair = false;
  single.slots = sm_count_cached();
  single.m_tiles = 0;
  for (int i = 0; i < nrows; ++i) single.m_tiles += (rows[i] + G_M - 1) / G_M;
  single.tiles = single.m_tiles * single.n_tiles;
  const double c256 = plan_splits(&single, G_SPLIT_MAX_TILES);
  // 128-token tiles: twice the tiles (the weight decoded twice as often per token), for
  // launches that would otherwise leave SMs idle or split K
  GemmPlan narrow = single;
  narrow.tile_n = G_NMAX / 2;
  narrow.n_tiles = (n + narrow.tile_n - 1) / narrow.tile_n;
  narrow.tiles = narrow.m_tiles * narrow.n_tiles;
  const double c128 = plan_splits(&narrow, G_SPLIT_MAX_TILES);
  const int tn_env = tile_n_env();
  const bool use128 = tn_env == 128 || (tn_env == 0 && c128 < 0.95 * c256);
  if (use128) single = narrow;
  const double c_single = use128 ? c128 : c256;
  // a forced token tile width (STEW_NF4_TILE_N) also keeps automatic plans on single CTAs
  const int mode = tn_env != 0 && pair_mode_env() != 1 ? 0 : pair_mode_env();
  const int64_t pslots = mode == 0 ? 0 : pair_slots_cached();
  if (pslots <= 0) return force_splits(single);
  // Pair tiles are near MMA-bound, so the tokens are dealt evenly over the fewest 512-token
  // tiles (a multiple of 32 each; e.g. 1311 tokens: 448 + 448 + 415, not 512 + 512 + 287):
  // the longest unit of a wave is what the launch waits for.
  GemmPlan pair = single;
  pair.n_tiles = (n + G_PAIR_TILE_N - 1) / G_PAIR_TILE_N;
  pair.tile_n = G_PAIR_TILE_N;
  pair.pair = true;
  pair.slots = pslots;
  pair.m_tiles = 0;
  for (int i = 0; i < nrows; ++i) pair.m_tiles += (rows[i] + 2 * G_M - 1) / (2 * G_M);
  pair.tiles = pair.m_tiles * pair.n_tiles;
  const double c_pair = plan_splits(&pair, G_SPLIT_MAX_TILES / 2);
  if (pair.n_tiles > 0) {
    const int64_t even = ((n + pair.n_tiles - 1) / pair.n_tiles + 31) / 32 * 32;
    pair.tile_n = int32_t(even < G_PAIR_TILE_N ? even : G_PAIR_TILE_N);
  }
  // automatic: pairs when the model puts them 5 % ahead of single CTAs
  GemmPlan chosen = (mode == 1 || c_pair < 0.95 * c_single) ? pair : single;
  return force_splits(chosen);
}

// Workspace of a split launch: the counter region, then one fp32 partial tile per K range
// and CTA tile [cta tiles][splits][256 tokens (a pair: 512)][128] (the last range of a tile
// to finish leaves its slot unused).
static int64_t plan_work_bytes(const GemmPlan& p) {
  if (p.splits <= 1) return 0;
  const int64_t cta_tiles = p.pair ? 2 * p.tiles : p.tiles;
  const int64_t acc_t = p.pair ? acc_tokens<true>() : acc_tokens<false>();
  return G_SPLIT_CNT_BYTES + cta_tiles * p.splits * int64_t(G_M) * acc_t * int64_t(sizeof(float));
}

// Token rows of the activation tile one CTA loads per stage.
static uint32_t act_box_rows(const GemmPlan& p) { return p.pair ? G_NMAX / 2 : uint32_t(p.tile_n); }

template <bool BWD, bool SPLIT, bool MULTI, bool PAIR, bool GLU = false>
static int launch_variant(unsigned grid, const CUtensorMap (&ta)[G_MAX_W], const CUtensorMap (&tw)[G_MAX_W],
                          const GemmArgs& g, cudaStream_t s) {
  int st = set_smem_attr<BWD, SPLIT, MULTI, PAIR, GLU>();
  if (st != NF4B_OK) return st;
  if (!PAIR) {
    NF4B_CUDA_TRY(launch_pdl(nf4_gemm_kernel<BWD, SPLIT, MULTI, PAIR, GLU>, dim3(grid), dim3(G_THREADS),
                             size_t(Smem<PAIR>::ALLOC), s, ta[0], ta[1], ta[2], tw[0], tw[1], tw[2], g));
  } else {
    PairLaunch pl(grid, s, pdl_enabled(s));
    NF4B_CUDA_TRY(cudaLaunchKernelEx(&pl.cfg, nf4_gemm_kernel<BWD, SPLIT, MULTI, PAIR, GLU>, ta[0], ta[1],
                                     ta[2], tw[0], tw[1], tw[2], g));
  }
  return NF4B_OK;
}

// Test hook (nf4b_test_drop_split_ticket): the work unit that the next split-K launch of this
// process skips the ticket of; -1 when unarmed.
static std::atomic<int> g_drop_ticket_unit{-1};

// One persistent CTA per SM, or one 2-CTA cluster per pair slot (at most one per work unit).
// glu: forward, a SwiGLU forward (gate and up as weights 0 and 1, one tile holding both);
// backward, the dX of down with the SwiGLU backward in its epilogue.
template <bool BWD>
static int launch_gemm(const GemmPlan& p, const CUtensorMap (&ta)[G_MAX_W], const CUtensorMap (&tw)[G_MAX_W],
                       GemmArgs g, void* work, int64_t work_bytes, cudaStream_t s, bool glu = false) {
  GemmPlan q = p;
  if (work == nullptr) q.splits = 1;
  NF4B_RETURN_IF(q.tiles * q.splits > 0x7FFFFFFFll, NF4B_ERR_UNSUPPORTED);
  if (q.splits > 1) {
    NF4B_RETURN_IF(work_bytes < plan_work_bytes(q), NF4B_ERR_INVALID_ARG);
    NF4B_RETURN_IF(!aligned(work, 256), NF4B_ERR_ALIGNMENT);
    g.ws_cnt = static_cast<int32_t*>(work);
    g.ws_part = reinterpret_cast<float*>(static_cast<uint8_t*>(work) + G_SPLIT_CNT_BYTES);
  }
  g.m_tiles = int32_t(q.m_tiles);
  g.n_tiles = int32_t(q.n_tiles);
  g.splits = q.splits;
  g.nk = q.nk;
  g.k16 = 1u << 16;
  g.tile_n = q.tile_n;
  g.drop_ticket_unit = q.splits > 1 ? g_drop_ticket_unit.exchange(-1) : -1;
  const int64_t units = q.tiles * q.splits;
  const int64_t slots = units < q.slots ? units : q.slots;
  const unsigned grid = unsigned(q.pair ? 2 * slots : slots);
  // backward launches with one unit per CTA (pair) at most (forward ones measured no faster)
  g.epi_decode = (BWD && units <= q.slots) ? 1 : 0;
  g.red_staged = red_staged_env();
  const bool split = q.splits > 1;
  const bool multi = g.nw > 1 && !glu;
  int st;
  if (glu) {
    if (q.pair)
      st = split ? launch_variant<BWD, true, false, true, true>(grid, ta, tw, g, s)
                 : launch_variant<BWD, false, false, true, true>(grid, ta, tw, g, s);
    else
      st = split ? launch_variant<BWD, true, false, false, true>(grid, ta, tw, g, s)
                 : launch_variant<BWD, false, false, false, true>(grid, ta, tw, g, s);
  } else if (q.pair) {
    if (multi)
      st = split ? launch_variant<BWD, true, true, true>(grid, ta, tw, g, s)
                 : launch_variant<BWD, false, true, true>(grid, ta, tw, g, s);
    else
      st = split ? launch_variant<BWD, true, false, true>(grid, ta, tw, g, s)
                 : launch_variant<BWD, false, false, true>(grid, ta, tw, g, s);
  } else {
    if (multi)
      st = split ? launch_variant<BWD, true, true, false>(grid, ta, tw, g, s)
                 : launch_variant<BWD, false, true, false>(grid, ta, tw, g, s);
    else
      st = split ? launch_variant<BWD, true, false, false>(grid, ta, tw, g, s)
                 : launch_variant<BWD, false, false, false>(grid, ta, tw, g, s);
  }
  if (st != NF4B_OK) return st;
  return launch_status(BWD ? "nf4_gemm_kernel<bwd> launch" : "nf4_gemm_kernel<fwd> launch");
}

// Validates the shared part of the forward/backward arguments.
static int gemm_common_checks(const void* act, const uint8_t* packed, const nf4b_qstate* qs,
                              const void* out, int64_t n, int64_t in_f, int64_t out_f,
                              int32_t* log2_bs) {
  NF4B_RETURN_IF(!act || !packed || !qs || !out || !qs->code, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(n < 0 || in_f <= 0 || out_f <= 0, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(in_f % G_K != 0 || out_f % G_K != 0, NF4B_ERR_UNSUPPORTED);
  NF4B_RETURN_IF(in_f > (1 << 24) || out_f > (1 << 24) || n > (int64_t(1) << 31),
                 NF4B_ERR_UNSUPPORTED);
  const int lb = ilog2_exact(qs->blocksize);
  NF4B_RETURN_IF(lb < 5 || lb > 8, NF4B_ERR_UNSUPPORTED);
  // nested == 2 (the unpack's contracted-scale debug form) has no fused-GEMM counterpart
  NF4B_RETURN_IF(qs->nested < 0 || qs->nested > 2, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(qs->nested == 2, NF4B_ERR_UNSUPPORTED);
  if (qs->nested) {
    NF4B_RETURN_IF(!qs->absmax8 || !qs->code2 || !qs->absmax2 || !qs->offset, NF4B_ERR_INVALID_ARG);
    NF4B_RETURN_IF(qs->blocksize2 != 256, NF4B_ERR_UNSUPPORTED);
  } else {
    NF4B_RETURN_IF(!qs->absmax32, NF4B_ERR_INVALID_ARG);
  }
  NF4B_RETURN_IF(!aligned(act, 16) || !aligned(packed, 16) || !aligned(out, 4),
                 NF4B_ERR_ALIGNMENT);
  *log2_bs = lb;
  return NF4B_OK;
}

static void fill_qstate_args(GemmW* w, const nf4b_qstate* qs, int32_t log2_bs) {
  w->absmax8 = qs->absmax8;
  w->absmax32 = qs->absmax32;
  w->code2 = qs->code2;
  w->absmax2 = qs->absmax2;
  w->offset = qs->offset;
  w->code = qs->code;
  w->log2_bs = log2_bs;
  w->nested = qs->nested ? 1 : 0;
}

// Global tile boundaries of the weights (tiles of 128 rows, 256 for pairs): unused entries
// stay past every tile.
static void set_m_end(GemmArgs* g, const int64_t* rows, int nw, bool pair) {
  const int64_t tr = pair ? 2 * G_M : G_M;
  int64_t acc = 0;
  for (int i = 0; i < G_MAX_W; ++i) {
    if (i < nw) acc += (rows[i] + tr - 1) / tr;
    g->m_end[i] = i < nw ? int32_t(acc) : 0x7FFFFFFF;
  }
  g->nw = nw;
}

int lora_project16_multi(const void* const* act, const void* const* w, int64_t w_stride_r,
                         int64_t w_stride_k, void* const* out, const int64_t* kdim, int n_jobs,
                         int64_t n, cudaStream_t s);  // lora.cu

}  // namespace nf4b

using namespace nf4b;

extern "C" int64_t nf4b_linear_work_bytes(int64_t n, int64_t in_features, int64_t out_features,
                                          int32_t backward) {
  if (n <= 0 || in_features <= 0 || out_features <= 0) return 0;
  if (check_device() != NF4B_OK) return -1;
  const int64_t rows = backward ? in_features : out_features;
  return plan_work_bytes(plan_gemm(n, &rows, 1, backward ? out_features : in_features));
}

extern "C" int64_t nf4b_linear_group_work_bytes(int64_t n, int64_t in_features,
                                                const int64_t* out_features, int32_t n_items) {
  if (n <= 0 || in_features <= 0 || !out_features || n_items < 1 || n_items > G_MAX_W) return 0;
  if (check_device() != NF4B_OK) return -1;
  return plan_work_bytes(plan_gemm(n, out_features, n_items, in_features));
}

extern "C" int nf4b_linear_fwd_group(const void* x, int64_t n, int64_t in_features,
                                     const nf4b_linear_item* items, int32_t n_items, void* work,
                                     int64_t work_bytes, void* stream) {
  NF4B_RETURN_IF(!items || n_items < 1, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(n_items > G_MAX_W, NF4B_ERR_UNSUPPORTED);
  int32_t lb[G_MAX_W];
  for (int i = 0; i < n_items; ++i) {
    const nf4b_linear_item& it = items[i];
    int st = gemm_common_checks(x, it.packed, it.qs, it.y, n, in_features, it.out_features, &lb[i]);
    if (st != NF4B_OK) return st;
    if (it.lora) {
      NF4B_RETURN_IF(it.lora->rank != 16, NF4B_ERR_UNSUPPORTED);
      NF4B_RETURN_IF(!it.lora->a || !it.lora->b || !it.lora->xa, NF4B_ERR_INVALID_ARG);
      NF4B_RETURN_IF(!aligned(it.lora->a, 16) || !aligned(it.lora->b, 16) || !aligned(it.lora->xa, 16),
                     NF4B_ERR_ALIGNMENT);
    }
  }
  if (n == 0) return NF4B_OK;
  int st = check_device();
  if (st != NF4B_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int64_t rows[G_MAX_W];
  for (int i = 0; i < n_items; ++i) rows[i] = items[i].out_features;
  const GemmPlan plan = plan_gemm(n, rows, n_items, in_features);
  CUtensorMap ta[G_MAX_W], tw[G_MAX_W];
  st = make_tmap_2d(&ta[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, uint64_t(in_features), uint64_t(n),
                    uint64_t(in_features) * 2, G_K, act_box_rows(plan), CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != NF4B_OK) return st;
  ta[1] = ta[2] = ta[0];
  GemmArgs g{};
  // the adapters' rank-16 projections, batched into one launch
  const void* pj_act[G_MAX_W];
  const void* pj_w[G_MAX_W];
  void* pj_out[G_MAX_W];
  int64_t pj_k[G_MAX_W];
  int npj = 0;
  for (int i = 0; i < n_items; ++i) {
    const nf4b_linear_item& it = items[i];
    st = make_tmap_2d(&tw[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, it.packed, uint64_t(in_features / 2),
                      uint64_t(it.out_features), uint64_t(in_features / 2), G_K / 2, G_M,
                      CU_TENSOR_MAP_SWIZZLE_32B);
    if (st != NF4B_OK) return st;
    GemmW& w = g.w[i];
    fill_qstate_args(&w, it.qs, lb[i]);
    w.bias = static_cast<const __half*>(it.bias);
    w.out = static_cast<__half*>(it.y);
    w.out_f = it.out_features;
    if (it.lora) {
      // X A^T of every adapter of the group: one launch below
      pj_act[npj] = x;
      pj_w[npj] = it.lora->a;
      pj_out[npj] = it.lora->xa;
      pj_k[npj] = in_features;
      ++npj;
      w.has_lora = 1;
      w.lora_w = static_cast<const __half*>(it.lora->b);
      w.lora_t = static_cast<const __half*>(it.lora->xa);
      w.lora_scale = it.lora->scale;
    }
  }
  if (npj > 0) {
    st = lora_project16_multi(pj_act, pj_w, in_features, 1, pj_out, pj_k, npj, n, s);
    if (st != NF4B_OK) return st;
  }
  for (int i = n_items; i < G_MAX_W; ++i) tw[i] = tw[0];  // unused kernel parameters
  set_m_end(&g, rows, n_items, plan.pair);
  for (int i = 0; i < G_MAX_W; ++i) g.k_end[i] = 0x7FFFFFFF;
  g.n = n;
  g.in_f = in_features;
  return launch_gemm<false>(plan, ta, tw, g, work, work_bytes, s);
}

extern "C" int nf4b_linear_fwd_ws(const void* x, const uint8_t* packed, const nf4b_qstate* qs,
                                  const void* bias, const nf4b_lora* lora, void* y, int64_t n,
                                  int64_t in_features, int64_t out_features, void* work,
                                  int64_t work_bytes, void* stream) {
  const nf4b_linear_item it{packed, qs, bias, lora, y, out_features};
  return nf4b_linear_fwd_group(x, n, in_features, &it, 1, work, work_bytes, stream);
}

extern "C" int nf4b_linear_fwd(const void* x, const uint8_t* packed, const nf4b_qstate* qs,
                               const void* bias, const nf4b_lora* lora, void* y, int64_t n,
                               int64_t in_features, int64_t out_features, void* stream) {
  return nf4b_linear_fwd_ws(x, packed, qs, bias, lora, y, n, in_features, out_features, nullptr, 0,
                            stream);
}

// ------------------------------------------------------------ SwiGLU forward
// Tiles of 64 features of gate and of up (128 operand rows), so the plan is that of one weight
// of 2 x out rows.
static GemmPlan plan_swiglu(int64_t n, int64_t in_features, int64_t out_features) {
  const int64_t rows = 2 * out_features;
  return plan_gemm(n, &rows, 1, in_features);
}

extern "C" int64_t nf4b_linear_swiglu_work_bytes(int64_t n, int64_t in_features, int64_t out_features) {
  if (n <= 0 || in_features <= 0 || out_features <= 0) return 0;
  if (check_device() != NF4B_OK) return -1;
  return plan_work_bytes(plan_swiglu(n, in_features, out_features));
}

extern "C" int nf4b_linear_fwd_swiglu(const void* x, int64_t n, int64_t in_features, const uint8_t* gate_packed,
                                      const nf4b_qstate* gate_qs, const uint8_t* up_packed,
                                      const nf4b_qstate* up_qs, void* gate_out, void* up_out, void* m_out,
                                      int64_t out_features, void* work, int64_t work_bytes, void* stream) {
  int32_t lb[2];
  int st = gemm_common_checks(x, gate_packed, gate_qs, gate_out, n, in_features, out_features, &lb[0]);
  if (st != NF4B_OK) return st;
  st = gemm_common_checks(x, up_packed, up_qs, up_out, n, in_features, out_features, &lb[1]);
  if (st != NF4B_OK) return st;
  NF4B_RETURN_IF(!m_out, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(!aligned(m_out, 4), NF4B_ERR_ALIGNMENT);
  if (n == 0) return NF4B_OK;
  st = check_device();
  if (st != NF4B_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const GemmPlan plan = plan_swiglu(n, in_features, out_features);
  CUtensorMap ta[G_MAX_W], tw[G_MAX_W];
  st = make_tmap_2d(&ta[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, uint64_t(in_features), uint64_t(n),
                    uint64_t(in_features) * 2, G_K, act_box_rows(plan), CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != NF4B_OK) return st;
  ta[1] = ta[2] = ta[0];
  // 64-row boxes: a stage holds 64 rows of gate, then the same 64 rows of up
  const uint8_t* packed[2] = {gate_packed, up_packed};
  for (int i = 0; i < 2; ++i) {
    st = make_tmap_2d(&tw[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, packed[i], uint64_t(in_features / 2),
                      uint64_t(out_features), uint64_t(in_features / 2), G_K / 2, G_M / 2, CU_TENSOR_MAP_SWIZZLE_32B);
    if (st != NF4B_OK) return st;
  }
  tw[2] = tw[0];
  GemmArgs g{};
  const nf4b_qstate* qs[2] = {gate_qs, up_qs};
  void* outs[2] = {gate_out, up_out};
  for (int i = 0; i < 2; ++i) {
    GemmW& w = g.w[i];
    fill_qstate_args(&w, qs[i], lb[i]);
    w.out = static_cast<__half*>(outs[i]);
    w.out_f = out_features;
  }
  const int64_t rows = 2 * out_features;
  set_m_end(&g, &rows, 1, plan.pair);
  g.nw = 2;  // both weights' code tables are loaded
  for (int i = 0; i < G_MAX_W; ++i) g.k_end[i] = 0x7FFFFFFF;
  g.n = n;
  g.in_f = in_features;
  g.glu_out = static_cast<__half*>(m_out);
  return launch_gemm<false>(plan, ta, tw, g, work, work_bytes, s, true);
}

extern "C" int64_t nf4b_linear_bwd_group_work_bytes(int64_t n, int64_t in_features,
                                                    const int64_t* out_features, int32_t n_items) {
  if (n <= 0 || in_features <= 0 || !out_features || n_items < 1 || n_items > G_MAX_W) return 0;
  if (check_device() != NF4B_OK) return -1;
  int64_t kdim = 0;
  for (int i = 0; i < n_items; ++i) kdim += out_features[i];
  return plan_work_bytes(plan_gemm(n, &in_features, 1, kdim));
}

extern "C" int nf4b_linear_bwd_dx_group(const nf4b_linear_bwd_item* items, int32_t n_items, void* dx,
                                        int64_t n, int64_t in_features, void* work,
                                        int64_t work_bytes, void* stream) {
  NF4B_RETURN_IF(!items || n_items < 1, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(n_items > G_MAX_W, NF4B_ERR_UNSUPPORTED);
  int32_t lb[G_MAX_W];
  int64_t kdim = 0;
  for (int i = 0; i < n_items; ++i) {
    const nf4b_linear_bwd_item& it = items[i];
    int st = gemm_common_checks(it.dy, it.packed, it.qs, dx, n, in_features, it.out_features, &lb[i]);
    if (st != NF4B_OK) return st;
    if (it.lora) {
      NF4B_RETURN_IF(it.lora->rank != 16, NF4B_ERR_UNSUPPORTED);
      NF4B_RETURN_IF(!it.lora->a || !it.lora->b || !it.dyb, NF4B_ERR_INVALID_ARG);
      NF4B_RETURN_IF(!aligned(it.lora->a, 16) || !aligned(it.lora->b, 16) || !aligned(it.dyb, 16),
                     NF4B_ERR_ALIGNMENT);
    }
    kdim += it.out_features;
  }
  NF4B_RETURN_IF(kdim / G_K > 0x7FFFFFFFll, NF4B_ERR_UNSUPPORTED);
  if (n == 0) return NF4B_OK;
  int st = check_device();
  if (st != NF4B_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const GemmPlan plan = plan_gemm(n, &in_features, 1, kdim);
  CUtensorMap ta[G_MAX_W], tw[G_MAX_W];
  GemmArgs g{};
  // the adapters' rank-16 projections, batched into one launch
  const void* pj_act[G_MAX_W];
  const void* pj_w[G_MAX_W];
  void* pj_out[G_MAX_W];
  int64_t pj_k[G_MAX_W];
  int npj = 0;
  int64_t kacc = 0;
  for (int i = 0; i < n_items; ++i) {
    const nf4b_linear_bwd_item& it = items[i];
    st = make_tmap_2d(&ta[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, it.dy, uint64_t(it.out_features),
                      uint64_t(n), uint64_t(it.out_features) * 2, G_K, act_box_rows(plan),
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != NF4B_OK) return st;
    st = make_tmap_2d(&tw[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, it.packed, uint64_t(in_features / 2),
                      uint64_t(it.out_features), uint64_t(in_features / 2), G_M / 2, G_K,
                      CU_TENSOR_MAP_SWIZZLE_64B);
    if (st != NF4B_OK) return st;
    GemmW& w = g.w[i];
    fill_qstate_args(&w, it.qs, lb[i]);
    w.out = static_cast<__half*>(dx);
    w.out_f = it.out_features;
    if (it.lora) {
      // dY B: B is [out, 16] row-major -> element (r, k=o) at o*16 + r; every adapter of the
      // group in one launch below
      pj_act[npj] = it.dy;
      pj_w[npj] = it.lora->b;
      pj_out[npj] = it.dyb;
      pj_k[npj] = it.out_features;
      ++npj;
      w.has_lora = 1;
      w.lora_w = static_cast<const __half*>(it.lora->a);
      w.lora_t = static_cast<const __half*>(it.dyb);
      w.lora_scale = it.lora->scale;
    }
    kacc += it.out_features / G_K;
    g.k_end[i] = int32_t(kacc);
  }
  if (npj > 0) {
    st = lora_project16_multi(pj_act, pj_w, 1, 16, pj_out, pj_k, npj, n, s);
    if (st != NF4B_OK) return st;
  }
  for (int i = n_items; i < G_MAX_W; ++i) {
    ta[i] = ta[0];  // unused kernel parameters
    tw[i] = tw[0];
    g.k_end[i] = 0x7FFFFFFF;
  }
  set_m_end(&g, &in_features, 1, plan.pair);  // all weights share the M side (the in features)
  g.nw = n_items;
  g.n = n;
  g.in_f = in_features;
  return launch_gemm<true>(plan, ta, tw, g, work, work_bytes, s);
}

extern "C" int nf4b_linear_bwd_dx_swiglu(const void* dy, const uint8_t* packed, const nf4b_qstate* qs,
                                         const void* gate, const void* up, void* dgate, void* dup, int64_t n,
                                         int64_t in_features, int64_t out_features, void* work,
                                         int64_t work_bytes, void* stream) {
  int32_t lb = 0;
  int st = gemm_common_checks(dy, packed, qs, dgate, n, in_features, out_features, &lb);
  if (st != NF4B_OK) return st;
  NF4B_RETURN_IF(!gate || !up || !dup, NF4B_ERR_INVALID_ARG);
  NF4B_RETURN_IF(!aligned(gate, 4) || !aligned(up, 4) || !aligned(dup, 4), NF4B_ERR_ALIGNMENT);
  if (n == 0) return NF4B_OK;
  st = check_device();
  if (st != NF4B_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the plan of the plain dX launch of this weight (same tiles, same K ranges)
  const GemmPlan plan = plan_gemm(n, &in_features, 1, out_features);
  CUtensorMap ta[G_MAX_W], tw[G_MAX_W];
  st = make_tmap_2d(&ta[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, dy, uint64_t(out_features), uint64_t(n),
                    uint64_t(out_features) * 2, G_K, act_box_rows(plan), CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != NF4B_OK) return st;
  st = make_tmap_2d(&tw[0], CU_TENSOR_MAP_DATA_TYPE_UINT8, packed, uint64_t(in_features / 2), uint64_t(out_features),
                    uint64_t(in_features / 2), G_M / 2, G_K, CU_TENSOR_MAP_SWIZZLE_64B);
  if (st != NF4B_OK) return st;
  ta[1] = ta[2] = ta[0];
  tw[1] = tw[2] = tw[0];
  GemmArgs g{};
  fill_qstate_args(&g.w[0], qs, lb);
  g.w[0].out = static_cast<__half*>(dgate);  // not written: the epilogue writes dgate / dup
  g.w[0].out_f = out_features;
  g.k_end[0] = int32_t(out_features / G_K);
  for (int i = 1; i < G_MAX_W; ++i) g.k_end[i] = 0x7FFFFFFF;
  set_m_end(&g, &in_features, 1, plan.pair);
  g.n = n;
  g.in_f = in_features;
  g.glu_g = static_cast<const __half*>(gate);
  g.glu_u = static_cast<const __half*>(up);
  g.glu_dg = static_cast<__half*>(dgate);
  g.glu_du = static_cast<__half*>(dup);
  return launch_gemm<true>(plan, ta, tw, g, work, work_bytes, s, true);
}

extern "C" int nf4b_linear_bwd_dx_ws(const void* dy, const uint8_t* packed, const nf4b_qstate* qs,
                                     const nf4b_lora* lora, void* dyb, void* dx, int64_t n,
                                     int64_t in_features, int64_t out_features, void* work,
                                     int64_t work_bytes, void* stream) {
  const nf4b_linear_bwd_item it{dy, packed, qs, lora, dyb, out_features};
  return nf4b_linear_bwd_dx_group(&it, 1, dx, n, in_features, work, work_bytes, stream);
}

extern "C" int nf4b_linear_bwd_dx(const void* dy, const uint8_t* packed, const nf4b_qstate* qs,
                                  const nf4b_lora* lora, void* dyb, void* dx, int64_t n,
                                  int64_t in_features, int64_t out_features, void* stream) {
  return nf4b_linear_bwd_dx_ws(dy, packed, qs, lora, dyb, dx, n, in_features, out_features, nullptr,
                               0, stream);
}

extern "C" int nf4b_gemm_error_flag(int* value, int reset) {
  NF4B_RETURN_IF(value == nullptr, NF4B_ERR_INVALID_ARG);
  NF4B_CUDA_TRY(cudaMemcpyFromSymbol(value, g_gemm_error, sizeof(int)));
  if (reset) {
    const int zero = 0;
    NF4B_CUDA_TRY(cudaMemcpyToSymbol(g_gemm_error, &zero, sizeof(int)));
  }
  return NF4B_OK;
}

extern "C" int nf4b_test_drop_split_ticket(int32_t unit) {
  NF4B_RETURN_IF(unit < 0, NF4B_ERR_INVALID_ARG);
  g_drop_ticket_unit.store(unit);
  return NF4B_OK;
}

extern "C" int nf4b_gemm_geometry(int* sms, int* pair_slots) {
  NF4B_RETURN_IF(sms == nullptr || pair_slots == nullptr, NF4B_ERR_INVALID_ARG);
  const int st = check_device();
  if (st != NF4B_OK) return st;
  *sms = sm_count_cached();
  *pair_slots = pair_slots_cached();
  return NF4B_OK;
}
