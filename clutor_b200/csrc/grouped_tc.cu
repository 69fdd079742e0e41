// Batched expert products on the 5th-generation tensor cores (tcgen05, accumulators in TMEM) for Q8_0 experts: the
// gate/up and down products of the reference's batched block (c/src/forward.c:1197-1201) as grouped GEMMs.
//
// Work: a tile is one expert, 256 weight rows and up to 32 of the expert's tokens (dispatch order). For gate/up the 256
// rows are gate rows [128m, 128m+128) (matrix 0) and the up rows of the same range (matrix 1); for down, down rows
// [256m, 256m+128) and [256m+128, 256m+256). A persistent CTA per SM walks the tiles round-robin; its warps specialise:
//   warp 8  (one lane) TMA-loads the raw Q8_0 weights, 128 rows x 256 elements (272 bytes a row) per box, into a ring
//           of shared-memory stages, running ahead of the dequantization across tiles;
//   warps 0-7  one weight row per thread (warps 0-3 matrix 0, 4-7 matrix 1): per 64-element atom they read their row's
//           bytes from the stage and write the dequantized weights into TMEM as two fp16 planes, hi = fp16(q*d) and
//           lo = fp16(q*d - hi) (half2 arithmetic: exact products, one rounding each), as the A operand of the MMAs;
//           at the end of a tile they read the accumulators (epilogue);
//   warp 10 (one lane) TMA-loads the tokens' activations (fp16 hi/lo planes, 64 x 16 boxes, 128-byte swizzle) as one
//           operand of 2N rows, [x hi | x lo];
//   warps 9 and 11 (one lane each; matrix 0 and matrix 1) issue per 16-element K step two MMAs, A hi and A lo (from
//           TMEM) times [x hi | x lo] (shared memory), into an fp32 TMEM accumulator of 128 rows x 2N, whose two halves the
//           epilogue adds: (w hi + w lo) * (x hi + x lo) in two instructions. An M=128, K=16 MMA takes about 45 cycles
//           whatever its N up to 64, so at a few tokens an expert the number of MMAs, not their width, bounds the loop.
// Products accurate to about 2^-22, so the result stays within 1e-6 relative of the reference's fp32 float path
// (c/src/quant.c:889-902) instead of the ~4e-4 that single fp16 operands give. Every hand-off is an mbarrier (TMA
// completion, tcgen05.commit, or warp arrivals); every wait is bounded and a timeout sets the error flag.
// Epilogue: gate/up -> SwiGLU -> hg as fp16 hi/lo planes (the down product's activations); down -> hd fp32.
#include <cuda.h>
#include <cuda_fp16.h>

#include <cstring>

#include "common.cuh"
#include "decode.cuh"
#include "tcgen05.cuh"

namespace clb {

namespace {

constexpr int DQ_WARPS = 8;                         // dequantizing warps, one weight row per thread
constexpr int W_RAW = DQ_WARPS, W_MMA0 = DQ_WARPS + 1, W_ACT = DQ_WARPS + 2, W_MMA1 = DQ_WARPS + 3;
constexpr int TC_THREADS = 32 * (DQ_WARPS + 4);
constexpr int TC_NT = 32;                           // tokens per accumulator tile
constexpr int RAW_STAGES = 5;
constexpr uint32_t CHUNK_BYTES = 272;               // 256 elements of Q8_0 (8 blocks of 34 bytes)
constexpr uint32_t RAW_STAGE = 128 * CHUNK_BYTES;   // one matrix's 128 rows of one chunk
constexpr int B_STAGES = 4;
constexpr uint32_t B_TILE = TC_NT * 128;            // up to 32 tokens x 64 fp16, 128-byte swizzle
constexpr uint32_t B_STAGE = 2 * B_TILE;            // hi rows [0, NT), lo rows [NT, 2 NT)
constexpr int A_STAGES = 3;
// TMEM columns: accumulators (2 NT columns: x hi products, then x lo products) of matrix 0 at [0, 64) and matrix 1 at
// [64, 128); A stage j at 128 + 128 j as [matrix 0 hi: 32][matrix 0 lo: 32][matrix 1 hi: 32][matrix 1 lo: 32] (64 fp16
// of K per row, two per column).
constexpr uint32_t ACC_COLS = 4 * TC_NT, A_COLS = 128, TMEM_COLS = 512;
static_assert(ACC_COLS + A_STAGES * A_COLS <= TMEM_COLS, "TMEM budget");
constexpr int N_BARS = 2 * RAW_STAGES + 2 * B_STAGES + 2 * A_STAGES + 3;
constexpr uint32_t SMEM_BYTES = RAW_STAGES * RAW_STAGE + B_STAGES * B_STAGE + 8 * N_BARS + 16 + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

// 2-D tiled TMA load of one box into shared memory, completing on `bar`.
CLB_DEV void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
               ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
               : "memory");
}

// The 4 bytes at byte offset `off` of a 272-byte chunk held as 68 little-endian words (off is a constant once unrolled).
CLB_DEV uint32_t word_at(const uint32_t (&w)[68], int off) {
  const int i = off >> 2, sh = off & 3;
  return sh == 0 ? w[i] : __byte_perm(w[i], w[i + 1], 0x3210 + 0x1111 * sh);
}

CLB_DEV __half2 as_half2(uint32_t v) {
  __half2 h;
  memcpy(&h, &v, 4);
  return h;
}
CLB_DEV uint32_t as_u32(__half2 h) {
  uint32_t v;
  memcpy(&v, &h, 4);
  return v;
}

// Four int8 values (one word) times an fp16 scale: the exact products rounded once to fp16 (hi) and the rounded remainders
// (lo), as two half2 pairs each. int8 q -> fp16 exactly: the bits of 1024 + (q + 128), minus 1152.
CLB_DEV void dequant4(uint32_t qw, __half2 d2, uint32_t &hi01, uint32_t &hi23, uint32_t &lo01, uint32_t &lo23) {
  const uint32_t u = qw ^ 0x80808080u;
  const __half2 bias = __half2half2(__ushort_as_half(0x6480));   // 1152
  const __half2 q01 = __hsub2(as_half2(__byte_perm(u, 0x64u, 0x4140)), bias);
  const __half2 q23 = __hsub2(as_half2(__byte_perm(u, 0x64u, 0x4342)), bias);
  const __half2 h01 = __hmul2(q01, d2), h23 = __hmul2(q23, d2);
  hi01 = as_u32(h01);
  hi23 = as_u32(h23);
  lo01 = as_u32(__hfma2(q01, d2, __hneg2(h01)));
  lo23 = as_u32(__hfma2(q23, d2, __hneg2(h23)));
}

// Q8_0 block b (0..7) of a 272-byte chunk as 16 columns of packed fp16 pairs, hi and lo planes.
CLB_DEV void dequant_block(const uint32_t (&w)[68], int b, uint32_t (&hi)[16], uint32_t (&lo)[16]) {
  const uint32_t dw = w[(34 * b) >> 2];   // the block's fp16 scale at byte 34b (2-byte aligned)
  const __half2 d2 = __half2half2(__ushort_as_half(static_cast<unsigned short>(((34 * b) & 3) == 0 ? (dw & 0xffffu) : (dw >> 16))));
#pragma unroll
  for (int i = 0; i < 8; ++i) dequant4(word_at(w, 34 * b + 2 + 4 * i), d2, hi[2 * i], hi[2 * i + 1], lo[2 * i], lo[2 * i + 1]);
}

// Calls f(e, m, pos0, nt) for this CTA's tiles: expert e, row tile m, tokens at dispatch positions [pos0, pos0 + nt).
// Every role of the CTA walks the same sequence. Stops (false) as soon as f fails.
template <class F>
CLB_DEV bool for_each_tile(const BatchArgs &a, int MT, F &&f) {
  const int TK = a.T * a.K;
  for (int w = blockIdx.x; w < a.NE * MT; w += gridDim.x) {
    const int e = w / MT, m = w - e * MT;
    const int n_e = a.counts[e], p0 = a.offsets[e];
    if (n_e <= 0 || p0 < 0 || p0 + n_e > TK) continue;
    for (int n0 = 0; n0 < n_e; n0 += TC_NT)
      if (!f(e, m, p0 + n0, min(TC_NT, n_e - n0))) return false;
  }
  return true;
}

}  // namespace

template <bool GATEUP>
__global__ void __launch_bounds__(TC_THREADS, 1)
    q80_group_tc_kernel(const BatchArgs a, const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                        const __grid_constant__ CUtensorMap tm_bh, const __grid_constant__ CUtensorMap tm_bl) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *raw = smem, *bst = smem + RAW_STAGES * RAW_STAGE;
  uint64_t *raw_full = reinterpret_cast<uint64_t *>(bst + B_STAGES * B_STAGE);   // [RAW_STAGES] weights landed
  uint64_t *raw_free = raw_full + RAW_STAGES;   // [RAW_STAGES] read by the 4 warps of its matrix
  uint64_t *b_full = raw_free + RAW_STAGES;     // [B_STAGES] activations landed
  uint64_t *b_free = b_full + B_STAGES;         // [B_STAGES] their MMAs done (both MMA warps)
  uint64_t *a_full = b_free + B_STAGES;         // [A_STAGES] TMEM A stage written by the 8 dequantizing warps
  uint64_t *a_free = a_full + A_STAGES;         // [A_STAGES] its MMAs done (both MMA warps)
  uint64_t *acc_full = a_free + A_STAGES;       // a tile's MMAs done (both MMA warps)
  uint64_t *acc_free = acc_full + 1;            // the accumulators read out by the 8 warps
  uint64_t *mma_done = acc_free + 1;            // every MMA the CTA issued has completed
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int MT = GATEUP ? a.FF / 128 : a.E / 256;
  const int nchunk = (GATEUP ? a.E : a.FF) / 256;
  const int rows_e = GATEUP ? a.FF : a.E;       // weight rows per expert

  if (threadIdx.x == 0) {
    for (int i = 0; i < RAW_STAGES; ++i) { mbar_init(&raw_full[i], 1); mbar_init(&raw_free[i], 4); }
    for (int i = 0; i < B_STAGES; ++i) { mbar_init(&b_full[i], 1); mbar_init(&b_free[i], 2); }
    for (int i = 0; i < A_STAGES; ++i) { mbar_init(&a_full[i], DQ_WARPS); mbar_init(&a_free[i], 2); }
    mbar_init(acc_full, 2);
    mbar_init(acc_free, DQ_WARPS);
    mbar_init(mma_done, 2);
    fence_barrier_init();
  }
  if (warp == 0) tc::tmem_alloc(tmem_slot, TMEM_COLS);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == W_RAW) {
    if (lane == 0) {
      uint32_t u = 0;   // half-stages issued: (chunk, matrix) in order
      ok = for_each_tile(a, MT, [&](int e, int m, int, int) {
        for (int c = 0; c < nchunk; ++c) {
          for (int mA = 0; mA < 2; ++mA, ++u) {
            const uint32_t s = u % RAW_STAGES;
            if (u >= RAW_STAGES && !mbar_wait_bounded(&raw_free[s], (u / RAW_STAGES - 1) & 1)) return false;
            const int y = e * rows_e + (GATEUP ? 128 * m : 256 * m + 128 * mA);
            mbar_arrive_expect_tx(&raw_full[s], RAW_STAGE);
            tma_load_2d(raw + s * RAW_STAGE, mA ? &tm_w1 : &tm_w0, 34 * c, y, &raw_full[s]);
          }
        }
        return true;
      });
      // every copy issued has landed before the CTA exits (already so unless a wait above gave up)
      for (uint32_t v = u > RAW_STAGES ? u - RAW_STAGES : 0; v < u; ++v)
        if (!mbar_wait_bounded(&raw_full[v % RAW_STAGES], (v / RAW_STAGES) & 1)) ok = false;
    }
  } else if (warp == W_ACT) {
    if (lane == 0) {
      uint32_t t = 0;   // atoms issued
      ok = for_each_tile(a, MT, [&](int, int, int pos0, int nt) {
        const int NT = (nt + 15) & ~15;
        for (int c = 0; c < nchunk; ++c) {
          for (int at = 0; at < 4; ++at, ++t) {
            const uint32_t s = t % B_STAGES;
            if (t >= B_STAGES && !mbar_wait_bounded(&b_free[s], (t / B_STAGES - 1) & 1)) return false;
            mbar_arrive_expect_tx(&b_full[s], static_cast<uint32_t>(NT) * 256u);
            uint8_t *bs = bst + s * B_STAGE;
            for (int j = 0; j < NT / 16; ++j) {
              tma_load_2d(bs + 2048 * j, &tm_bh, 256 * c + 64 * at, pos0 + 16 * j, &b_full[s]);
              tma_load_2d(bs + 128 * NT + 2048 * j, &tm_bl, 256 * c + 64 * at, pos0 + 16 * j, &b_full[s]);
            }
          }
        }
        return true;
      });
      for (uint32_t v = t > B_STAGES ? t - B_STAGES : 0; v < t; ++v)
        if (!mbar_wait_bounded(&b_full[v % B_STAGES], (v / B_STAGES) & 1)) ok = false;
    }
  } else if (warp == W_MMA0 || warp == W_MMA1) {
    if (lane == 0) {
      const int mA = warp == W_MMA0 ? 0 : 1;
      const uint32_t acc = tmem + 2 * TC_NT * mA;
      uint32_t t = 0, it = 0;
      ok = for_each_tile(a, MT, [&](int, int, int, int nt) {
        const uint32_t idesc = tc::idesc_f16_f32(128, 2 * ((nt + 15) & ~15));
        if (it > 0 && !mbar_wait_bounded(acc_free, (it - 1) & 1)) return false;
        tc::fence_after_sync();
        for (int c = 0; c < nchunk; ++c) {
          for (int at = 0; at < 4; ++at, ++t) {
            const uint32_t sa = t % A_STAGES, sb = t % B_STAGES;
            if (!mbar_wait_bounded(&a_full[sa], (t / A_STAGES) & 1)) return false;
            if (!mbar_wait_bounded(&b_full[sb], (t / B_STAGES) & 1)) return false;
            tc::fence_after_sync();
            const uint64_t bdesc = tc::sw128_desc(smem_addr(bst + sb * B_STAGE));
            const uint32_t ah = tmem + ACC_COLS + A_COLS * sa + 64 * mA;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {   // K step: +8 TMEM columns of A, +32 bytes (2 descriptor units) of B
              tc::mma_f16_ts(acc, ah + 8 * kk, bdesc + 2 * kk, idesc, c != 0 || at != 0 || kk != 0);
              tc::mma_f16_ts(acc, ah + 32 + 8 * kk, bdesc + 2 * kk, idesc, true);
            }
            tc::commit(&a_free[sa]);
            tc::commit(&b_free[sb]);
          }
        }
        tc::commit(acc_full);
        ++it;
        return true;
      });
      tc::commit(mma_done);   // the TMEM is released only after every MMA issued has completed
      if (!mbar_wait_bounded(mma_done, 0)) ok = false;
    }
  } else {   // dequantizing warps
    const int mA = warp >> 2, q = warp & 3, r = 32 * q + lane;
    const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;
    uint32_t g = 0, t = 0, it = 0;   // chunks, atoms, tiles consumed
    ok = for_each_tile(a, MT, [&](int, int m, int pos0, int nt) {
      for (int c = 0; c < nchunk; ++c, ++g) {
        const uint32_t u = 2 * g + mA, s = u % RAW_STAGES;
        if (!mbar_wait_bounded(&raw_full[s], (u / RAW_STAGES) & 1)) return false;
        uint32_t w[68];
        const uint4 *src = reinterpret_cast<const uint4 *>(raw + s * RAW_STAGE + r * CHUNK_BYTES);
#pragma unroll
        for (int i = 0; i < 17; ++i) {
          const uint4 v = src[i];
          w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_free[s]);
#pragma unroll
        for (int at = 0; at < 4; ++at, ++t) {
          const uint32_t sa = t % A_STAGES;
          if (t >= A_STAGES && !mbar_wait_bounded(&a_free[sa], (t / A_STAGES - 1) & 1)) return false;
          tc::fence_after_sync();
          const uint32_t col = tmem + lane_base + ACC_COLS + A_COLS * sa + 64 * mA;
#pragma unroll
          for (int bb = 0; bb < 2; ++bb) {
            uint32_t hi[16], lo[16];
            dequant_block(w, 2 * at + bb, hi, lo);
            tc::st_x16(col + 16 * bb, hi);
            tc::st_x16(col + 32 + 16 * bb, lo);
          }
          tc::wait_st();
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[sa]);
        }
      }
      // epilogue: warps of matrix 0 take tokens [0, 16), those of matrix 1 [16, 32); each reads both accumulators, whose
      // column n holds the x hi products and column NT + n the x lo products of token n
      if (!mbar_wait_bounded(acc_full, it & 1)) return false;
      tc::fence_after_sync();
      const int c0 = 16 * mA, NT = (nt + 15) & ~15;
      float v0[16], v1[16];
      if (c0 < nt) {
        float l0[16], l1[16];
        tc::ld_x16(tmem + lane_base + c0, v0);
        tc::ld_x16(tmem + lane_base + NT + c0, l0);
        tc::ld_x16(tmem + lane_base + 2 * TC_NT + c0, v1);
        tc::ld_x16(tmem + lane_base + 2 * TC_NT + NT + c0, l1);
#pragma unroll
        for (int j = 0; j < 16; ++j) { v0[j] = __fadd_rn(v0[j], l0[j]); v1[j] = __fadd_rn(v1[j], l1[j]); }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_free);
      ++it;
      if (c0 < nt) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int n = c0 + j;
          if (n >= nt) break;
          const size_t pos = static_cast<size_t>(pos0 + n);
          if (GATEUP) {
            const float h = silu_mul(v0[j], v1[j]);
            const __half hh = __float2half_rn(h);
            const __half hl = __float2half_rn(__fsub_rn(h, __half2float(hh)));
            const size_t o = pos * a.FF + 128 * m + r;
            a.hgh[o] = hh;
            a.hgl[o] = hl;
          } else {
            const size_t o = pos * a.E + 256 * m + r;
            a.hd[o] = v0[j];
            a.hd[o + 128] = v1[j];
          }
        }
      }
      return true;
    });
    if (warp == 0 && lane == 0) {   // experts whose dispatch range is out of bounds are skipped; report them
      for (int e = blockIdx.x; e < a.NE; e += gridDim.x) {
        const int n_e = a.counts[e], p0 = a.offsets[e];
        if (n_e > 0 && (p0 < 0 || p0 + n_e > a.T * a.K)) set_error(a.err, ERR_BAD_EXPERT);
      }
    }
  }
  if (!ok) set_error(a.err, ERR_WAIT_COPY);
  if (warp < DQ_WARPS) tc::wait_st();   // nothing of this thread's in flight on the TMEM
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_dealloc(tmem, TMEM_COLS);
}

template __global__ void q80_group_tc_kernel<true>(const BatchArgs, const __grid_constant__ CUtensorMap, const __grid_constant__ CUtensorMap,
                                                   const __grid_constant__ CUtensorMap, const __grid_constant__ CUtensorMap);
template __global__ void q80_group_tc_kernel<false>(const BatchArgs, const __grid_constant__ CUtensorMap, const __grid_constant__ CUtensorMap,
                                                    const __grid_constant__ CUtensorMap, const __grid_constant__ CUtensorMap);

// Gathers the fp16 hi/lo planes of xn into dispatch order (row p = the token at dispatch position p).
__global__ void gather_x_kernel(const BatchArgs a) {
  const int p = blockIdx.x, t = a.pos_token[p];
  if (t < 0 || t >= a.T) { if (threadIdx.x == 0) set_error(a.err, ERR_BAD_EXPERT); return; }
  const uint4 *sh = reinterpret_cast<const uint4 *>(a.xh + static_cast<size_t>(t) * a.E);
  const uint4 *sl = reinterpret_cast<const uint4 *>(a.xl + static_cast<size_t>(t) * a.E);
  uint4 *dh = reinterpret_cast<uint4 *>(a.xdh + static_cast<size_t>(p) * a.E);
  uint4 *dl = reinterpret_cast<uint4 *>(a.xdl + static_cast<size_t>(p) * a.E);
  for (int i = threadIdx.x; i < a.E / 8; i += blockDim.x) { dh[i] = sh[i]; dl[i] = sl[i]; }
}

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *, const cuuint64_t *,
                                 const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess && p) fn = reinterpret_cast<EncodeTiled>(p);
  }
  return fn;
}

// A 2-D fp16 tensor map over a [rows x cols] row-major plane: boxes of 64 columns x 16 rows, 128-byte swizzle (the
// canonical K-major layout the MMAs read), zeros outside the tensor.
static bool encode_plane(CUtensorMap *m, const void *base, int rows, int cols) {
  const EncodeTiled fn = encoder();
  if (!fn) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {64, 16}, estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A 2-D map over Q8_0 weight rows [rows x row_bytes] (all experts' rows one after another), in 8-byte units: boxes of
// 272 bytes (one 256-element chunk) x 128 rows, no swizzle (rows land 272 bytes apart).
static bool encode_raw(CUtensorMap *m, const void *base, int rows, uint32_t row_bytes) {
  const EncodeTiled fn = encoder();
  if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes % CHUNK_BYTES)) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes / 8), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  const cuuint32_t box[2] = {CHUNK_BYTES / 8, 128}, estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool q80_tc_supported(const void *gate, const void *up, const void *down, int E, int FF) {
  const uintptr_t any = reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up) | reinterpret_cast<uintptr_t>(down);
  return (any & 15) == 0 && E % 256 == 0 && FF % 256 == 0 && E >= 256 && FF >= 256;
}

int launch_q80_tc(const BatchArgs &a, void *stream_, bool gateup) {
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  const int TK = a.T * a.K;
  CUtensorMap tw0, tw1, tbh, tbl;
  bool ok;
  if (gateup) {
    gather_x_kernel<<<TK, 256, 0, st>>>(a);
    ok = encode_raw(&tw0, a.gate, a.NE * a.FF, a.grb) && encode_raw(&tw1, a.up, a.NE * a.FF, a.grb) &&
         encode_plane(&tbh, a.xdh, TK, a.E) && encode_plane(&tbl, a.xdl, TK, a.E);
  } else {
    ok = encode_raw(&tw0, a.down, a.NE * a.E, a.drb) && encode_raw(&tw1, a.down, a.NE * a.E, a.drb) &&
         encode_plane(&tbh, a.hgh, TK, a.FF) && encode_plane(&tbl, a.hgl, TK, a.FF);
  }
  if (!ok) return static_cast<int>(cudaErrorInvalidValue);
  int dev = 0;
  cudaGetDevice(&dev);
  static int sms[64] = {};
  if (dev < 0 || dev >= 64) return static_cast<int>(cudaErrorInvalidDevice);
  if (!sms[dev]) {
    cudaFuncSetAttribute(q80_group_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    cudaFuncSetAttribute(q80_group_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  }
  const int tiles = a.NE * (gateup ? a.FF / 128 : a.E / 256);
  const int grid = tiles < sms[dev] ? tiles : sms[dev];
  if (gateup) q80_group_tc_kernel<true><<<grid, TC_THREADS, SMEM_BYTES, st>>>(a, tw0, tw1, tbh, tbl);
  else q80_group_tc_kernel<false><<<grid, TC_THREADS, SMEM_BYTES, st>>>(a, tw0, tw1, tbh, tbl);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace clb
