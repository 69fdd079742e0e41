// Steps of the whole-model forward pass that both the one-token kernel (fwd.cu) and the batched prompt kernels
// (prefill.cu) use: the embedding row and the rotary embedding of one head.
#pragma once
#include <cstdint>

#include "common.cuh"
#include "fwd.cuh"
#include "rowdot.cuh"

namespace clb {

// One row of the token embedding as floats, the reference's cl_dequant_row (c/src/quant.c:59-66, 87-105, 155-158).
CLB_DEV void embed_row(const FwdMat &m, int token, int E, float *y) {
  const uint8_t *row = m.p + static_cast<size_t>(token) * m.rb;
  for (int i = threadIdx.x; i < E; i += blockDim.x) {
    float v;
    if (m.type == T_Q4_K) {
      const uint8_t *b = row + 144 * (i / 256);
      const int e = i % 256, j = e / 64, hi = (e / 32) & 1, l = e % 32;
      int sc, mn;
      q4k_scale_min(b + 4, 2 * j + hi, sc, mn);
      const float d = f16_bits_to_f32(lds_u16(b)), dmin = f16_bits_to_f32(lds_u16(b + 2));
      const int q = hi ? (b[16 + 32 * j + l] >> 4) : (b[16 + 32 * j + l] & 15);
      v = __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q)), __fmul_rn(dmin, static_cast<float>(mn)));
    } else if (m.type == T_Q6_K) {
      const uint8_t *b = row + 210 * (i / 256);
      const int e = i % 256, n = e / 128, r = e % 128, part = r / 32, l = r % 32;
      const uint8_t *ql = b + 64 * n, *qh = b + 128 + 32 * n;
      const int8_t *sc = reinterpret_cast<const int8_t *>(b + 192) + 8 * n;
      const int lo = (part & 1) ? ql[l + 32] : ql[l];
      const int q = ((part < 2 ? (lo & 15) : (lo >> 4)) | (((qh[l] >> (2 * part)) & 3) << 4)) - 32;
      const float d = f16_bits_to_f32(lds_u16(b + 208));
      v = __fmul_rn(__fmul_rn(d, static_cast<float>(sc[l / 16 + 2 * part])), static_cast<float>(q));
    } else if (m.type == T_Q8_0) {
      const uint8_t *b = row + 34 * (i / 32);
      v = __fmul_rn(static_cast<float>(static_cast<int8_t>(b[2 + i % 32])), f16_bits_to_f32(lds_u16(b)));
    } else {   // F32
      v = reinterpret_cast<const float *>(row)[i];
    }
    y[i] = v;
  }
}

// Rotary embedding of one head held by a warp, EPL = hd / 32 elements per lane at i = lane + 32 e. NEOX pairs (i, i + hd/2)
// (c/src/forward.c:428-435) or adjacent pairs (2i, 2i + 1) (:420-426). The angle's cosine and sine come from tables the
// host filled with the reference's own expressions and C library (cosf / sinf of pos * powf(base, -2i / hd)): cs holds
// [hd / 2] cosines then [hd / 2] sines for this position (global or shared memory).
template <int EPL>
CLB_DEV void rope_warp(float (&v)[EPL], const float *cs, bool pairs) {
  constexpr int H = 16 * EPL;   // hd / 2
  const int lane = threadIdx.x & 31;
  if (!pairs) {
#pragma unroll
    for (int e = 0; e < EPL / 2; ++e) {
      const float c = cs[lane + 32 * e], s = cs[H + lane + 32 * e];
      const float a = v[e], b = v[e + EPL / 2];
      v[e] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
      v[e + EPL / 2] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    }
  } else {
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int i = lane + 32 * e;
      const float c = cs[i / 2], s = cs[H + i / 2];
      const float other = __shfl_xor_sync(FULL, v[e], 1);
      const float a = (i & 1) ? other : v[e], b = (i & 1) ? v[e] : other;
      v[e] = (i & 1) ? __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c)) : __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    }
  }
}

}  // namespace clb
