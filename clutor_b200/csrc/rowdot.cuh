// Warp-cooperative dot products of one GGUF-quantized weight row (in shared memory) with one activation vector, giving the
// reference's results bit for bit.
//
// K-quants (Q4_K, Q6_K) against Q8_K activations: a row of nblk 256-element blocks is split into 4*nblk "units" of 64
// elements (4 per block). Each lane computes the exact integer partial sums of its units with dp4a; the four lanes of a block
// add them (integer sums are exact in any order), the block's first lane forms the block's float term exactly as the
// reference does (c/src/quant.c:832-846: yd*(d*sumi - dmin*summs) for Q4_K, (d*yd)*sumi for Q6_K), and the terms are added
// in block order with one rounding each, which is the reference's float order. A row group is 4*nblk lanes (several rows per
// warp when that is below 32) or the whole warp (a lane then holds several units).
//
// Q8_0 against float activations: the reference's float path (c/src/quant.c:889-902): per 32-element block, s = sum of
// (q*d)*x in element order, then the row total adds the block sums in block order.
#pragma once
#include "common.cuh"

namespace clb {

constexpr unsigned FULL = 0xffffffffu;
constexpr int KQ_MAXI = 2;     // units per lane: rows up to 8 * 32 / 4 * 2 = 4096 wide
constexpr int Q80_MAXI = 4;    // Q8_0 blocks per lane: rows up to 4096 wide

// Byte offset of 16-byte chunk j of 256-block b in a swizzled Q8_K value array: chunk j sits at position j ^ (b & 7), so
// that eight lanes reading chunk j of eight consecutive blocks hit eight different groups of banks.
CLB_DEV int q8k_chunk_off(int b, int j, bool swz) { return 256 * b + 16 * (swz ? (j ^ (b & 7)) : j); }

// How a warp splits rows of `units` units into row groups.
struct RowShape {
  int LG;   // lanes per row group
  int RPW;  // row groups per warp
  int NI;   // units per lane
};
CLB_DEV RowShape row_shape(int units) {
  RowShape s;
  if (units <= 32) { s.LG = units; s.RPW = 32 / units; s.NI = 1; }
  else { s.LG = 32; s.RPW = 1; s.NI = (units + 31) / 32; }
  return s;
}

// Activation registers of one lane for K-quant units: 64 int8 values (16 words), the 4 group sums those units touch, and the
// block scale.
struct KQAct {
  int32_t q[KQ_MAXI][16];
  int32_t bs[KQ_MAXI][4];
  float d[KQ_MAXI];
};

// Loads unit u of a Q8_K activation vector (qs/d/bsums in shared memory) in the order the weight type's unit reads it.
CLB_DEV void load_kq_unit(uint32_t type, const int8_t *qs, const float *dd, const int16_t *bsums, int u, int32_t (&q)[16],
                          int32_t (&bs)[4], float &d) {
  const int blk = u >> 2, g = u & 3;
  const int8_t *base = qs + blk * 256;
  const int16_t *b16 = bsums + blk * 16;
  if (type == T_Q4_K) {       // elements 64g .. 64g+63: low nibbles then high nibbles of qs[32g .. 32g+31]
    const int4 *p = reinterpret_cast<const int4 *>(base + 64 * g);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int4 v = p[t];
      q[4 * t] = v.x; q[4 * t + 1] = v.y; q[4 * t + 2] = v.z; q[4 * t + 3] = v.w;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) bs[j] = b16[4 * g + j];
  } else {                    // Q6_K: half h = g/2, c = g%2 and c+2 of that half (elements 128h + 32c + l)
    const int h = g >> 1, cc = g & 1;
    const int4 *lo = reinterpret_cast<const int4 *>(base + 128 * h + 32 * cc);
    const int4 *hi = reinterpret_cast<const int4 *>(base + 128 * h + 32 * (cc + 2));
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int4 a = lo[t], b = hi[t];
      q[4 * t] = a.x; q[4 * t + 1] = a.y; q[4 * t + 2] = a.z; q[4 * t + 3] = a.w;
      q[8 + 4 * t] = b.x; q[8 + 4 * t + 1] = b.y; q[8 + 4 * t + 2] = b.z; q[8 + 4 * t + 3] = b.w;
    }
    const int g0 = 8 * h + 2 * cc;
    bs[0] = b16[g0]; bs[1] = b16[g0 + 1]; bs[2] = b16[g0 + 4]; bs[3] = b16[g0 + 5];
  }
  d = dd[blk];
}

CLB_DEV void load_kq_act(uint32_t type, const int8_t *qs, const float *dd, const int16_t *bsums, int nblk, RowShape rs,
                         int lane_in_grp, KQAct &a) {
#pragma unroll
  for (int i = 0; i < KQ_MAXI; ++i) {
    const int u = lane_in_grp + rs.LG * i;
    if (i < rs.NI && u < 4 * nblk) load_kq_unit(type, qs, dd, bsums, u, a.q[i], a.bs[i], a.d[i]);
  }
}

// Q4_K unit g of the block at blk (16-byte aligned): exact integer sum of scale*q*a and of min*bsum.
CLB_DEV void q4k_unit(const uint8_t *blk, int g, const int32_t (&q)[16], const int32_t (&bs)[4], int &sumi, int &summs) {
  const uint4 *p = reinterpret_cast<const uint4 *>(blk + 16 + 32 * g);
  const uint4 w0 = p[0], w1 = p[1];
  const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  int a = 0, c = 0;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    a = __dp4a(static_cast<int>(w[t] & 0x0F0F0F0Fu), q[t], a);
    c = __dp4a(static_cast<int>((w[t] >> 4) & 0x0F0F0F0Fu), q[8 + t], c);
  }
  int sc0, mn0, sc1, mn1;
  q4k_scale_min(blk + 4, 2 * g, sc0, mn0);
  q4k_scale_min(blk + 4, 2 * g + 1, sc1, mn1);
  sumi = sc0 * a + sc1 * c;
  summs = mn0 * (bs[0] + bs[1]) + mn1 * (bs[2] + bs[3]);
}

// Q6_K unit g of the block at blk (any alignment): values are 6-bit 0..63 taken as q+32, so each 16-group's sum is
// dot(v, a) - 32 * bsum, which is the reference's integer sum of (v-32)*a exactly.
CLB_DEV void q6k_unit(const uint8_t *blk, int g, const int32_t (&q)[16], const int32_t (&bs)[4], int &sumi) {
  const int h = g >> 1, cc = g & 1;
  const uint8_t *ql = blk + 64 * h + 32 * cc, *qh = blk + 128 + 32 * h;
  const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192);
  int lo0 = 0, lo1 = 0, hi0 = 0, hi1 = 0;
  const uint32_t sh_lo = 2 * cc, sh_hi = 2 * cc + 4;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const uint32_t l = lds_u32_unaligned(ql + 4 * t), hh = lds_u32_unaligned(qh + 4 * t);
    const int vlo = static_cast<int>((l & 0x0F0F0F0Fu) | (((hh >> sh_lo) & 0x03030303u) << 4));
    const int vhi = static_cast<int>(((l >> 4) & 0x0F0F0F0Fu) | (((hh >> sh_hi) & 0x03030303u) << 4));
    if (t < 4) { lo0 = __dp4a(vlo, q[t], lo0); hi0 = __dp4a(vhi, q[8 + t], hi0); }
    else { lo1 = __dp4a(vlo, q[t], lo1); hi1 = __dp4a(vhi, q[8 + t], hi1); }
  }
  const int g0 = 8 * h + 2 * cc;
  sumi = sc[g0] * (lo0 - 32 * bs[0]) + sc[g0 + 1] * (lo1 - 32 * bs[1]) + sc[g0 + 4] * (hi0 - 32 * bs[2]) +
         sc[g0 + 5] * (hi1 - 32 * bs[3]);
}

// One K-quant row (shared memory) times the lane's activation registers. All 32 lanes must call it with the same nblk and
// shape (warp-uniform control flow); `active` is false for a row group with no row. Returns the row's value in every lane of
// the group.
CLB_DEV float kq_row(uint32_t type, const uint8_t *row, int nblk, RowShape rs, int lane_in_grp, int grp_lane0,
                     const KQAct &a, bool active) {
  const uint32_t bb = type == T_Q4_K ? 144u : 210u;
  float t[KQ_MAXI];
#pragma unroll
  for (int i = 0; i < KQ_MAXI; ++i) {
    t[i] = 0.f;
    if (i < rs.NI) {
      const int u = lane_in_grp + rs.LG * i;
      const int blk = u >> 2, g = u & 3;
      const bool valid = active && u < 4 * nblk;
      int sumi = 0, summs = 0;
      const uint8_t *bp = row + blk * bb;
      if (valid) {
        if (type == T_Q4_K) q4k_unit(bp, g, a.q[i], a.bs[i], sumi, summs);
        else q6k_unit(bp, g, a.q[i], a.bs[i], sumi);
      }
      sumi += __shfl_xor_sync(FULL, sumi, 1);
      sumi += __shfl_xor_sync(FULL, sumi, 2);
      if (type == T_Q4_K) {
        summs += __shfl_xor_sync(FULL, summs, 1);
        summs += __shfl_xor_sync(FULL, summs, 2);
      }
      if (valid && g == 0) {
        if (type == T_Q4_K) {
          const float d = f16_bits_to_f32(lds_u16(bp)), dmin = f16_bits_to_f32(lds_u16(bp + 2));
          t[i] = __fmul_rn(a.d[i], __fsub_rn(__fmul_rn(d, static_cast<float>(sumi)), __fmul_rn(dmin, static_cast<float>(summs))));
        } else {
          const float d = f16_bits_to_f32(lds_u16(bp + 208));
          t[i] = __fmul_rn(__fmul_rn(d, a.d[i]), static_cast<float>(sumi));
        }
      }
    }
  }
  float sum = 0.f;
  for (int b = 0; b < nblk; ++b) {
    const int u = 4 * b, i = u / rs.LG;
    const float v = __shfl_sync(FULL, i == 0 ? t[0] : t[KQ_MAXI - 1], grp_lane0 + (u % rs.LG));
    sum = __fadd_rn(sum, v);
  }
  return sum;
}

// One Q8_0 row (shared memory, any alignment) times float activations xf (shared memory, 16-byte aligned): the reference's
// float path. Units are 32-element blocks; same calling rules as kq_row.
CLB_DEV float q80_row(const uint8_t *row, int nb32, RowShape rs, int lane_in_grp, int grp_lane0, const float *xf,
                      bool active) {
  float s[Q80_MAXI];
#pragma unroll
  for (int i = 0; i < Q80_MAXI; ++i) {
    s[i] = 0.f;
    const int b = lane_in_grp + rs.LG * i;
    if (i < rs.NI && active && b < nb32) {
      const uint8_t *bp = row + 34 * b;
      const float d = f16_bits_to_f32(lds_u16(bp));
      const float4 *x4 = reinterpret_cast<const float4 *>(xf + 32 * b);
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const uint32_t q4 = lds_u32_unaligned(bp + 2 + 4 * w);
        const float4 x = x4[w];
        acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int8_t>(q4 & 0xff)), d), x.x));
        acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int8_t>((q4 >> 8) & 0xff)), d), x.y));
        acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int8_t>((q4 >> 16) & 0xff)), d), x.z));
        acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int8_t>(q4 >> 24)), d), x.w));
      }
      s[i] = acc;
    }
  }
  float sum = 0.f;
  for (int b = 0; b < nb32; ++b) {
    const int i = b / rs.LG;
    float v = s[0];
#pragma unroll
    for (int j = 1; j < Q80_MAXI; ++j) v = i == j ? s[j] : v;
    sum = __fadd_rn(sum, __shfl_sync(FULL, v, grp_lane0 + (b % rs.LG)));
  }
  return sum;
}

// Q8_K quantization of n floats (shared memory) into qs/d/bsums (shared memory), one 256-block per warp at a time
// (c/src/quant.c:195-206): d = amax/127, q = roundf(x * (1/d)), bsums = sums of 16. Call from all threads of the block.
CLB_DEV void q8k_quantize_block(const float *x, int n, int8_t *qs, float *dd, int16_t *bsums, int warp, int nwarps,
                                int lane, bool swz = false) {
  for (int b = warp; b < n / 256; b += nwarps) {
    const float *v = x + 256 * b + 8 * lane;
    float vals[8];
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) { vals[j] = v[j]; amax = fmaxf(amax, fabsf(vals[j])); }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(FULL, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    int s = 0;
    uint32_t packed[2] = {0, 0};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int q = static_cast<int>(roundf(__fmul_rn(vals[j], id)));
      s += q;
      packed[j >> 2] |= (static_cast<uint32_t>(q) & 0xffu) << (8 * (j & 3));
    }
    reinterpret_cast<uint2 *>(qs + q8k_chunk_off(b, lane >> 1, swz) + 8 * (lane & 1))[0] = make_uint2(packed[0], packed[1]);
    s += __shfl_xor_sync(FULL, s, 1);
    if ((lane & 1) == 0) bsums[16 * b + lane / 2] = static_cast<int16_t>(s);
    if (lane == 0) dd[b] = d;
  }
}

// ---- one lane per 256-element block ---------------------------------------------------------------------------------------
// Activation registers for one whole block: 256 int8 values (64 words), the 16 group sums, the scale.
struct BlockAct {
  int32_t q[64];
  int32_t bs[16];
  float d;
};
// Loads 256-block blk of a swizzled Q8_K value array (q8k_chunk_off) with its group sums and scale.
CLB_DEV void load_block_act(const int8_t *qs, const float *dd, const int16_t *bsums, int blk, BlockAct &a) {
#pragma unroll
  for (int t = 0; t < 16; ++t) {
    const int4 v = *reinterpret_cast<const int4 *>(qs + q8k_chunk_off(blk, t, true));
    a.q[4 * t] = v.x; a.q[4 * t + 1] = v.y; a.q[4 * t + 2] = v.z; a.q[4 * t + 3] = v.w;
  }
  const int4 *b = reinterpret_cast<const int4 *>(bsums + 16 * blk);   // 16 int16 = two int4
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int4 v = b[t];
    const uint32_t w[4] = {static_cast<uint32_t>(v.x), static_cast<uint32_t>(v.y), static_cast<uint32_t>(v.z), static_cast<uint32_t>(v.w)};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      a.bs[8 * t + 2 * j] = static_cast<int16_t>(w[j] & 0xffffu);
      a.bs[8 * t + 2 * j + 1] = static_cast<int16_t>(w[j] >> 16);
    }
  }
  a.d = dd[blk];
}

CLB_DEV uint32_t lds_u32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }
CLB_DEV int byte_of(uint32_t w, int i) { return static_cast<int>((w >> (8 * i)) & 0xffu); }

// One Q4_K block (144 bytes at bp, 4-byte aligned) times a register block: the reference's term
// yd * (d * sumi - dmin * summs) with exact integer sums (c/src/quant.c:255-287, 832-846). The 12 packed scale bytes are
// unpacked with word operations: scales 0-3 / mins 0-3 are the low 6 bits of bytes 0-3 / 4-7; scales 4-7 / mins 4-7 are the
// low / high nibbles of bytes 8-11 with the top two bits of bytes 0-3 / 4-7 above them (ggml's layout, c/src/quant.c:36-52).
CLB_DEV float q4k_block(const uint8_t *bp, const BlockAct &a) {
  const uint32_t dm = lds_u32(bp), w0 = lds_u32(bp + 4), w1 = lds_u32(bp + 8), w2 = lds_u32(bp + 12);
  const uint32_t scA = w0 & 0x3f3f3f3fu, mnA = w1 & 0x3f3f3f3fu;
  const uint32_t scB = (w2 & 0x0f0f0f0fu) | (((w0 >> 6) & 0x03030303u) << 4);
  const uint32_t mnB = ((w2 >> 4) & 0x0f0f0f0fu) | (((w1 >> 6) & 0x03030303u) << 4);
  int sumi = 0;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint4 x0 = reinterpret_cast<const uint4 *>(bp + 16 + 32 * g)[0];
    const uint4 x1 = reinterpret_cast<const uint4 *>(bp + 16 + 32 * g)[1];
    const uint32_t w[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    int lo = 0, hi = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      lo = __dp4a(static_cast<int>(w[t] & 0x0f0f0f0fu), a.q[16 * g + t], lo);
      hi = __dp4a(static_cast<int>((w[t] >> 4) & 0x0f0f0f0fu), a.q[16 * g + 8 + t], hi);
    }
    const uint32_t sw = g < 2 ? scA : scB;
    sumi += byte_of(sw, 2 * (g & 1)) * lo + byte_of(sw, 2 * (g & 1) + 1) * hi;
  }
  int summs = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) summs += byte_of(j < 4 ? mnA : mnB, j & 3) * (a.bs[2 * j] + a.bs[2 * j + 1]);
  const float d = f16_bits_to_f32(static_cast<uint16_t>(dm & 0xffffu)), dmin = f16_bits_to_f32(static_cast<uint16_t>(dm >> 16));
  return __fmul_rn(a.d, __fsub_rn(__fmul_rn(d, static_cast<float>(sumi)), __fmul_rn(dmin, static_cast<float>(summs))));
}

// One Q6_K block (210 bytes at bp, any alignment) times a register block: the reference's term (d * yd) * sumi
// (c/src/quant.c:329-360). Element 128h + 32c + l takes a nibble of ql[64h + 32(c%2) + l] (low for c < 2) and bits 2c..2c+1
// of qh[32h + l]; the 6-bit value minus 32 is the weight. Each 16-group's dot is taken on the unsigned 6-bit values and
// corrected by 32 * (sum of the group's activations), which is the same integer.
CLB_DEV float q6k_block(const uint8_t *bp, const BlockAct &a) {
  int dot[16];
#pragma unroll
  for (int g = 0; g < 16; ++g) dot[g] = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const uint32_t L0 = lds_u32_unaligned(bp + 64 * h + 4 * t), L1 = lds_u32_unaligned(bp + 64 * h + 32 + 4 * t);
      const uint32_t H = lds_u32_unaligned(bp + 128 + 32 * h + 4 * t);
      const int v0 = static_cast<int>((L0 & 0x0f0f0f0fu) | ((H & 0x03030303u) << 4));
      const int v1 = static_cast<int>((L1 & 0x0f0f0f0fu) | (((H >> 2) & 0x03030303u) << 4));
      const int v2 = static_cast<int>(((L0 >> 4) & 0x0f0f0f0fu) | (((H >> 4) & 0x03030303u) << 4));
      const int v3 = static_cast<int>(((L1 >> 4) & 0x0f0f0f0fu) | (((H >> 6) & 0x03030303u) << 4));
      const int gq = t / 4;   // 16-group within each 32-element run
      dot[8 * h + gq] = __dp4a(v0, a.q[32 * h + t], dot[8 * h + gq]);
      dot[8 * h + 2 + gq] = __dp4a(v1, a.q[32 * h + 8 + t], dot[8 * h + 2 + gq]);
      dot[8 * h + 4 + gq] = __dp4a(v2, a.q[32 * h + 16 + t], dot[8 * h + 4 + gq]);
      dot[8 * h + 6 + gq] = __dp4a(v3, a.q[32 * h + 24 + t], dot[8 * h + 6 + gq]);
    }
  }
  const int8_t *sc = reinterpret_cast<const int8_t *>(bp + 192);
  int sumi = 0;
#pragma unroll
  for (int g = 0; g < 16; ++g) sumi += static_cast<int>(sc[g]) * (dot[g] - 32 * a.bs[g]);
  const float d = f16_bits_to_f32(lds_u16(bp + 208));
  return __fmul_rn(__fmul_rn(d, a.d), static_cast<float>(sumi));
}

CLB_DEV float kq_block(uint32_t type, const uint8_t *row, int blk, const BlockAct &a) {
  return type == T_Q4_K ? q4k_block(row + 144 * blk, a) : q6k_block(row + 210 * blk, a);
}

// The same two block terms with the activation block read from shared memory as it is needed (a swizzled Q8_K array:
// q8k_chunk_off) instead of held in registers: for kernels that use a block for one or two rows only, where 81 registers
// of activations would cost more than the shared-memory reads.
struct SmemAct {
  const int8_t *qs;      // swizzled values
  const int16_t *bsums;
  const float *dd;
};
CLB_DEV int4 act_chunk(const SmemAct &a, int blk, int j) {
  return *reinterpret_cast<const int4 *>(a.qs + q8k_chunk_off(blk, j, true));
}
// (The outer loops of these two stay rolled: kernels that run every phase once per layer are bound by fetching their
// code, not by these loops' overhead.)
template <bool COMPACT = true>
CLB_DEV float q4k_block_s(const uint8_t *bp, const SmemAct &a, int blk) {
  const uint32_t dm = lds_u32(bp), w0 = lds_u32(bp + 4), w1 = lds_u32(bp + 8), w2 = lds_u32(bp + 12);
  const uint32_t scA = w0 & 0x3f3f3f3fu, mnA = w1 & 0x3f3f3f3fu;
  const uint32_t scB = (w2 & 0x0f0f0f0fu) | (((w0 >> 6) & 0x03030303u) << 4);
  const uint32_t mnB = ((w2 >> 4) & 0x0f0f0f0fu) | (((w1 >> 6) & 0x03030303u) << 4);
  int sumi = 0;
#pragma unroll(COMPACT ? 1 : 4)
  for (int g = 0; g < 4; ++g) {
    const uint4 x0 = reinterpret_cast<const uint4 *>(bp + 16 + 32 * g)[0];
    const uint4 x1 = reinterpret_cast<const uint4 *>(bp + 16 + 32 * g)[1];
    const int4 c0 = act_chunk(a, blk, 4 * g), c1 = act_chunk(a, blk, 4 * g + 1), c2 = act_chunk(a, blk, 4 * g + 2),
               c3 = act_chunk(a, blk, 4 * g + 3);
    const int ql[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w}, qh[8] = {c2.x, c2.y, c2.z, c2.w, c3.x, c3.y, c3.z, c3.w};
    const uint32_t w[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    int lo = 0, hi = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      lo = __dp4a(static_cast<int>(w[t] & 0x0f0f0f0fu), ql[t], lo);
      hi = __dp4a(static_cast<int>((w[t] >> 4) & 0x0f0f0f0fu), qh[t], hi);
    }
    const uint32_t sw = g < 2 ? scA : scB;
    sumi += byte_of(sw, 2 * (g & 1)) * lo + byte_of(sw, 2 * (g & 1) + 1) * hi;
  }
  const int16_t *b16 = a.bsums + 16 * blk;
  int summs = 0;
#pragma unroll(COMPACT ? 1 : 8)
  for (int j = 0; j < 8; ++j) summs += byte_of(j < 4 ? mnA : mnB, j & 3) * (b16[2 * j] + b16[2 * j + 1]);
  const float d = f16_bits_to_f32(static_cast<uint16_t>(dm & 0xffffu)), dmin = f16_bits_to_f32(static_cast<uint16_t>(dm >> 16));
  return __fmul_rn(a.dd[blk], __fsub_rn(__fmul_rn(d, static_cast<float>(sumi)), __fmul_rn(dmin, static_cast<float>(summs))));
}
template <bool COMPACT = true>
CLB_DEV float q6k_block_s(const uint8_t *bp, const SmemAct &a, int blk) {
  const int8_t *sc = reinterpret_cast<const int8_t *>(bp + 192);
  const int16_t *b16 = a.bsums + 16 * blk;
  int sumi = 0;
#pragma unroll(COMPACT ? 1 : 2)
  for (int h = 0; h < 2; ++h) {
    int dot[8];
#pragma unroll
    for (int g = 0; g < 8; ++g) dot[g] = 0;
#pragma unroll
    for (int half = 0; half < 2; ++half) {   // t = 4 * half .. 4 * half + 3: one 16-group of each 32-element run
      const int4 a0 = act_chunk(a, blk, 8 * h + half), a1 = act_chunk(a, blk, 8 * h + 2 + half),
                 a2 = act_chunk(a, blk, 8 * h + 4 + half), a3 = act_chunk(a, blk, 8 * h + 6 + half);
      const int q0[4] = {a0.x, a0.y, a0.z, a0.w}, q1[4] = {a1.x, a1.y, a1.z, a1.w}, q2[4] = {a2.x, a2.y, a2.z, a2.w},
                q3[4] = {a3.x, a3.y, a3.z, a3.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = 4 * half + u;
        const uint32_t L0 = lds_u32_unaligned(bp + 64 * h + 4 * t), L1 = lds_u32_unaligned(bp + 64 * h + 32 + 4 * t);
        const uint32_t H = lds_u32_unaligned(bp + 128 + 32 * h + 4 * t);
        const int v0 = static_cast<int>((L0 & 0x0f0f0f0fu) | ((H & 0x03030303u) << 4));
        const int v1 = static_cast<int>((L1 & 0x0f0f0f0fu) | (((H >> 2) & 0x03030303u) << 4));
        const int v2 = static_cast<int>(((L0 >> 4) & 0x0f0f0f0fu) | (((H >> 4) & 0x03030303u) << 4));
        const int v3 = static_cast<int>(((L1 >> 4) & 0x0f0f0f0fu) | (((H >> 6) & 0x03030303u) << 4));
        dot[half] = __dp4a(v0, q0[u], dot[half]);
        dot[2 + half] = __dp4a(v1, q1[u], dot[2 + half]);
        dot[4 + half] = __dp4a(v2, q2[u], dot[4 + half]);
        dot[6 + half] = __dp4a(v3, q3[u], dot[6 + half]);
      }
    }
#pragma unroll
    for (int g = 0; g < 8; ++g) sumi += static_cast<int>(sc[8 * h + g]) * (dot[g] - 32 * b16[8 * h + g]);
  }
  const float d = f16_bits_to_f32(lds_u16(bp + 208));
  return __fmul_rn(__fmul_rn(d, a.dd[blk]), static_cast<float>(sumi));
}
// Weight block blk of `row` times activation block ablk (the swizzle key of the array: its index in the whole array).
// COMPACT keeps the outer loops rolled (small code for code run once per phase); else they are unrolled (hot loops).
template <bool COMPACT = true>
CLB_DEV float kq_block_s(uint32_t type, const uint8_t *row, int blk, const SmemAct &a, int ablk) {
  return type == T_Q4_K ? q4k_block_s<COMPACT>(row + 144 * blk, a, ablk) : q6k_block_s<COMPACT>(row + 210 * blk, a, ablk);
}

// Q8_K quantization of nblocks 256-blocks of floats in global memory (written by other CTAs; read through L2) into shared
// qs/d/bsums. Each warp takes blocks warp, warp + nwarps, ...; a lane issues the loads of up to BATCH blocks before the
// first reduction, so their round trips overlap.
template <int BATCH = 4>
CLB_DEV void q8k_quantize_global(const float *src, int nblocks, int8_t *qs, float *dd, int16_t *bsums, int warp, int nwarps,
                                 int lane, bool swz = false) {
  for (int b0 = warp; b0 < nblocks; b0 += BATCH * nwarps) {
    float4 v[BATCH][2];
#pragma unroll
    for (int j = 0; j < BATCH; ++j) {
      const int b = b0 + j * nwarps;
      if (b < nblocks) {
        const float4 *p = reinterpret_cast<const float4 *>(src + 256 * b + 8 * lane);
        v[j][0] = __ldcg(p);
        v[j][1] = __ldcg(p + 1);
      }
    }
#pragma unroll
    for (int j = 0; j < BATCH; ++j) {
      const int b = b0 + j * nwarps;
      if (b >= nblocks) break;
      const float vals[8] = {v[j][0].x, v[j][0].y, v[j][0].z, v[j][0].w, v[j][1].x, v[j][1].y, v[j][1].z, v[j][1].w};
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(vals[i]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(FULL, amax, o));
      const float d = __fdiv_rn(amax, 127.0f);
      const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
      int s = 0;
      uint32_t packed[2] = {0, 0};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int q = static_cast<int>(roundf(__fmul_rn(vals[i], id)));
        s += q;
        packed[i >> 2] |= (static_cast<uint32_t>(q) & 0xffu) << (8 * (i & 3));
      }
      reinterpret_cast<uint2 *>(qs + q8k_chunk_off(b, lane >> 1, swz) + 8 * (lane & 1))[0] = make_uint2(packed[0], packed[1]);
      s += __shfl_xor_sync(FULL, s, 1);
      if ((lane & 1) == 0) bsums[16 * b + lane / 2] = static_cast<int16_t>(s);
      if (lane == 0) dd[b] = d;
    }
  }
}

}  // namespace clb
