// Register-resident NF4 decode used inside the fused GEMMs.
//
// For one quantization block with scale s, the 16 possible outputs are
// T[i] = fp16_rn(code[i] * s) (fp32 multiply, one rounding -- exactly the value
// the reference unpack produces, solution/nf4.py:45-50).  The table is kept in
// 8 registers as two byte planes (low bytes L0..L3, high bytes H0..H3 of
// T[0..15]); a 4-nibble group is looked up with byte permutes:
//   entries 0..7 : prmt(L0, L1, nibbles)          (valid where nibble < 8)
//   entries 8..15: prmt(L2, L3, nibbles & 0x7777) (valid where nibble >= 8)
//   pick per byte by nibble bit 3, then interleave low/high planes into half2.
// Cost: 11 integer ops per 4 values + 32 ops per table (16 fmul, 8 cvt, 8 prmt); the
// multiply-high form below moves 5 of every 23 per word to the FMA pipe.
#pragma once

#include "common.cuh"

namespace nf4b {

struct Nf4Table {
  uint32_t l0, l1, l2, l3, h0, h1, h2, h3;
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ Nf4Table make_table(const float (&code)[16], float scale) {
  uint32_t p[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    p[i] = pack_half2(__fmul_rn(code[2 * i], scale), __fmul_rn(code[2 * i + 1], scale));
  Nf4Table t;
  t.l0 = prmt(p[0], p[1], 0x6420u);
  t.h0 = prmt(p[0], p[1], 0x7531u);
  t.l1 = prmt(p[2], p[3], 0x6420u);
  t.h1 = prmt(p[2], p[3], 0x7531u);
  t.l2 = prmt(p[4], p[5], 0x6420u);
  t.h2 = prmt(p[4], p[5], 0x7531u);
  t.l3 = prmt(p[6], p[7], 0x6420u);
  t.h3 = prmt(p[6], p[7], 0x7531u);
  return t;
}

// Two packed bytes (low 16 bits of s: byte0 = bits 0-7, high nibble first) ->
// two half2 words holding the 4 values in memory order.
__device__ __forceinline__ uint2 lookup4(const Nf4Table& t, uint32_t s) {
  const uint32_t m = s & 0x7777u;
  const uint32_t sel = ((s >> 1) & 0x4444u) | 0x3210u;
  const uint32_t lo = prmt(prmt(t.l0, t.l1, s), prmt(t.l2, t.l3, m), sel);
  const uint32_t hi = prmt(prmt(t.h0, t.h1, s), prmt(t.h2, t.h3, m), sel);
  return make_uint2(prmt(lo, hi, 0x4051u), prmt(lo, hi, 0x6273u));
}

// lookup4 with the nibble masks precomputed: m = s & 0x7777, sel = ((s >> 1) & 0x4444) | 0x3210
// (only the low 16 bits of each operand are read).
__device__ __forceinline__ uint2 lookup4_pre(const Nf4Table& t, uint32_t s, uint32_t m, uint32_t sel) {
  const uint32_t lo = prmt(prmt(t.l0, t.l1, s), prmt(t.l2, t.l3, m), sel);
  const uint32_t hi = prmt(prmt(t.h0, t.h1, s), prmt(t.h2, t.h3, m), sel);
  return make_uint2(prmt(lo, hi, 0x4051u), prmt(lo, hi, 0x6273u));
}

// As decode_word_f16, with the masks made once per word and its right shifts done as integer
// multiply-high, (x * 2^(32-s)) >> 32, which issue on the FMA pipe and leave the ALU pipe --
// the one the byte permutes saturate -- 18 instead of 23 instructions per word.  k16 = 1 << 16
// and k31 = 1 << 31 arrive as run-time values so the compiler keeps the multiplies.
__device__ __forceinline__ uint4 decode_word_f16_mh(const Nf4Table& t, uint32_t w, uint32_t k16,
                                                    uint32_t k31) {
  const uint32_t m = w & 0x77777777u;
  const uint32_t sel = (__umulhi(w, k31) & 0x44444444u) | 0x32103210u;
  const uint2 a = lookup4_pre(t, w, m, sel);
  const uint2 b = lookup4_pre(t, __umulhi(w, k16), __umulhi(m, k16), __umulhi(sel, k16));
  return make_uint4(a.x, a.y, b.x, b.y);
}

// One packed 32-bit word (8 values) -> 16 bytes of fp16 in memory order.
__device__ __forceinline__ uint4 decode_word_f16(const Nf4Table& t, uint32_t w) {
  const uint2 a = lookup4(t, w);
  const uint2 b = lookup4(t, w >> 16);
  return make_uint4(a.x, a.y, b.x, b.y);
}

}  // namespace nf4b
