// Batched expert products on the 5th-generation tensor cores (tcgen05, accumulators in TMEM) as grouped GEMMs: the
// gate/up and down products of the reference's batched block (c/src/forward.c:1197-1201) for Q8_0 and Q4_K experts.
//
// Work: a tile is one expert, 256 weight rows and up to NT of the expert's tokens (dispatch order; NT = 32 for Q8_0, 64
// for Q4_K). For gate/up the 256 rows are gate rows [128m, 128m+128) (matrix 0) and the up rows of the same range
// (matrix 1); for down, down rows [256m, 256m+128) and [256m+128, 256m+256). A persistent CTA per SM walks the tiles
// round-robin; its warps specialise:
//   warp 8  (one lane) TMA-loads the raw weights, 128 rows x one 256-element chunk (Q8_0: 272 bytes a row, eight blocks;
//           Q4_K: 144 bytes, one block) per box, into a ring of shared-memory stages, running ahead across tiles;
//   warps 0-7  one weight row per thread (warps 0-3 matrix 0, 4-7 matrix 1): per 64-element atom they read their row's
//           bytes from the stage and write the dequantized weights w into TMEM as two fp16 planes, hi = fp16(w) and
//           lo = fp16(w - hi), the A operand of the MMAs. Q8_0: w = q*d (half2 arithmetic: exact products, one rounding
//           each). Q4_K: w = d*sc*q - dmin*mn, the block's whole dequantized weight (c/src/quant.c:54-68) -- so the min
//           term needs no second product -- formed in fp32 (d*sc*q is exact, one rounding for the difference); at the
//           end of a tile they read the accumulators (epilogue);
//   warp 10 (one lane) TMA-loads the tokens' activations as one operand of 2N rows, [x hi | x lo] (fp16, 64 x 16 boxes,
//           128-byte swizzle): Q8_0 experts take xn itself (the reference's float path, c/src/quant.c:889-902); K-quant
//           experts take the value of the reference's Q8_K activations, yd * q8 (c/src/quant.h:22), so the product is
//           the reference's integer dot sum_b yd (d * sumi - dmin * summs) (c/src/quant.c:255-287) up to rounding;
//   warps 9 and 11 (one lane each; matrix 0 and matrix 1) issue per 16-element K step two MMAs, A hi and A lo (from
//           TMEM) times [x hi | x lo] (shared memory), into an fp32 TMEM accumulator of 128 rows x 2N, whose two halves
//           the epilogue adds: (w hi + w lo) * (x hi + x lo) in two instructions. An M=128, K=16 MMA takes about 45
//           cycles whatever its N up to 64, so at a few tokens an expert the number of MMAs, not their width, counts.
// Products accurate to about 2^-22, so the result stays within about 1e-6 relative of the reference's. Every hand-off is
// an mbarrier (TMA completion, tcgen05.commit, or warp arrivals); every wait is bounded and a timeout sets the error flag.
// Epilogue: gate/up -> SwiGLU -> hg (fp32, and for Q8_0 down also as fp16 hi/lo planes, its activations); down -> hd.
//
// Dispatch positions at or past the number of dispatched slots (offsets[NE]; fewer than T * K on an expert-parallel
// expert side, where other GPUs hold some of the experts) hold no data: no kernel here reads them for a result.
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
constexpr uint32_t A_COLS = 128, TMEM_COLS = 512;   // A stage: [m0 hi 32][m0 lo 32][m1 hi 32][m1 lo 32] TMEM columns

// Per weight type: bytes of a row's 256-element chunk, tokens per tile, ring depths, and how the x hi / x lo products
// are kept. Q8_0 (STACK): an accumulator of 2 NT columns per matrix, x hi products then x lo products (one MMA of width
// 2 NT per A plane: at a few tokens an expert the count of MMAs counts), matrix 0 at [0, 2NT), matrix 1 at [2NT, 4NT).
// Q4_K: 128 tokens a tile, so each weight is dequantized once per 128 tokens; an accumulator of NT columns per matrix
// ([0, NT) and [NT, 2NT)) that takes w hi x hi, w hi x lo and w lo x hi in turn (w lo x lo, about 2^-22 of the product, is
// left out). A stage j at ACC_COLS + 128 j (64 fp16 of K per row, two per column).
template <uint32_t WT>
struct TcShape {
  static constexpr bool STACK = WT == T_Q8_0;
  static constexpr uint32_t CHUNK = WT == T_Q8_0 ? 272u : 144u;
  static constexpr int NT = WT == T_Q8_0 ? 32 : 128;
  static constexpr int RAW_STAGES = WT == T_Q8_0 ? 5 : 6;
  static constexpr int B_STAGES = WT == T_Q8_0 ? 4 : 3;   // activation stages, one 64-column atom each
  static constexpr uint32_t RAW_STAGE = 128 * CHUNK;
  static constexpr uint32_t B_TILE = NT * 128;      // NT tokens x 64 fp16, 128-byte swizzle
  static constexpr uint32_t B_STAGE = 2 * B_TILE;   // hi rows [0, NT), lo rows [NT, 2 NT)
  static constexpr uint32_t ACC_COLS = (STACK ? 4 : 2) * NT;
  static constexpr int A_STAGES = static_cast<int>((TMEM_COLS - ACC_COLS) / A_COLS);
  static constexpr int N_BARS = 2 * RAW_STAGES + 2 * B_STAGES + 2 * A_STAGES + 3;
  static constexpr uint32_t SMEM = RAW_STAGES * RAW_STAGE + B_STAGES * B_STAGE + 8 * N_BARS + 16 + 1024;
  static_assert(A_STAGES >= 2, "TMEM budget");
  static_assert(SMEM + (3 * 1024 + 1) * 4 <= 232448, "shared memory budget (with the work list)");
  static_assert(CHUNK % 16 == 0, "TMA boxes are 16-byte multiples");
};

// 2-D tiled TMA load of one box into shared memory, completing on `bar`.
CLB_DEV void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
               ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
               : "memory");
}

// The 4 bytes at byte offset `off` of a chunk held as little-endian words (off is a constant once unrolled).
template <int NW>
CLB_DEV uint32_t word_at(const uint32_t (&w)[NW], int off) {
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

// Dequantization of one atom (64 values), its words read from shared memory per atom so the atom loop can stay rolled and
// its code small. Q8_0: blocks 2 at and 2 at + 1 of a 272-byte chunk (68 bytes as 17 words), piece bb of them, as 16
// columns of packed fp16 pairs, hi and lo planes.
CLB_DEV void dequant_q80_atom(const uint32_t (&w)[17], int bb, uint32_t (&hi)[16], uint32_t (&lo)[16]) {
  const uint32_t dw = w[(34 * bb) >> 2];
  const __half2 d2 = __half2half2(__ushort_as_half(static_cast<unsigned short>(((34 * bb) & 3) == 0 ? (dw & 0xffffu) : (dw >> 16))));
#pragma unroll
  for (int i = 0; i < 8; ++i) dequant4(word_at(w, 34 * bb + 2 + 4 * i), d2, hi[2 * i], hi[2 * i + 1], lo[2 * i], lo[2 * i + 1]);
}

// SwiGLU through one out-of-line copy: the epilogue's unrolled loop would otherwise hold sixteen copies of the double
// exponential, code that runs once per tile and so is fetched again for every tile.
__device__ __noinline__ float silu_mul_once(float g, float u) { return silu_mul(g, u); }

CLB_DEV float half_bits(uint32_t bits16) { return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16))); }
CLB_DEV uint32_t pack_half2(float a, float b) { return as_u32(__floats2half2_rn(a, b)); }   // a in the low half

// Q4_K: sub-block j (0..7) of a block from its header words (d, dmin, 12 scale bytes) and the 8 quant words of its
// 64-value group (quant bytes 32*(j/2) .. +31), as 16 columns of packed fp16 pairs of w = d*sc*q - dmin*mn, hi and lo
// planes. Sub-block j's values are the low (j even) or high (j odd) nibbles; scales and mins unpack as in
// c/src/quant.c:36-40.
CLB_DEV void dequant_q4k_atom(const uint32_t (&hdr)[4], const uint32_t (&qw8)[8], int j, uint32_t (&hi)[16], uint32_t (&lo)[16]) {
  const float d = half_bits(hdr[0] & 0xffffu), dmin = half_bits(hdr[0] >> 16);
  auto sbyte = [&](int i) -> int {   // scale byte i (0..11)
    const uint32_t wd = i < 4 ? hdr[1] : i < 8 ? hdr[2] : hdr[3];
    return static_cast<int>((wd >> (8 * (i & 3))) & 0xffu);
  };
  int sc, mn;
  if (j < 4) {
    sc = sbyte(j) & 63;
    mn = sbyte(j + 4) & 63;
  } else {
    sc = (sbyte(j + 4) & 15) | ((sbyte(j - 4) >> 6) << 4);
    mn = (sbyte(j + 4) >> 4) | ((sbyte(j) >> 6) << 4);
  }
  const float a1 = __fmul_rn(d, static_cast<float>(sc)), a0 = __fmul_rn(dmin, static_cast<float>(mn));   // both exact
  // w = a1*q - a0 with one rounding, two values per instruction: q comes in as the float 2^23 + q (its bits 0x4B000000 | q,
  // one byte permute), a1*(2^23 + q) - a1*2^23 = a1*q exactly (at most 21 significant bits), then - a0 rounds once
  const float2 A1 = make_float2(a1, a1), NA1M = make_float2(-a1 * 8388608.0f, -a1 * 8388608.0f), NA0 = make_float2(-a0, -a0);
  const uint32_t magic = 0x4B000000u;
  const int shift = (j & 1) ? 4 : 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t m = (qw8[i] >> shift) & 0x0F0F0F0Fu;   // the four values of this word, one per byte
    const float2 q01 = make_float2(__uint_as_float(__byte_perm(m, magic, 0x7440)), __uint_as_float(__byte_perm(m, magic, 0x7441)));
    const float2 q23 = make_float2(__uint_as_float(__byte_perm(m, magic, 0x7442)), __uint_as_float(__byte_perm(m, magic, 0x7443)));
    const float2 v01 = fadd2(ffma2(A1, q01, NA1M), NA0), v23 = fadd2(ffma2(A1, q23, NA1M), NA0);
    const __half2 h01 = __floats2half2_rn(v01.x, v01.y), h23 = __floats2half2_rn(v23.x, v23.y);
    const float2 l01 = fsub2(v01, __half22float2(h01)), l23 = fsub2(v23, __half22float2(h23));   // exact remainders
    hi[2 * i] = as_u32(h01);
    hi[2 * i + 1] = as_u32(h23);
    lo[2 * i] = as_u32(__floats2half2_rn(l01.x, l01.y));
    lo[2 * i + 1] = as_u32(__floats2half2_rn(l23.x, l23.y));
  }
}


// The CTA's work items: (expert e, row tile m, token chunk) for every expert with tokens, numbered expert by expert, row tile
// by row tile, the chunks of a tile consecutive (so CTAs running side by side share a weight tile in L2); item w goes to CTA
// w mod gridDim. pre[e] = the items of experts before e (pre[NE] = all), cnt / off = each expert's tokens and first dispatch
// position (experts with an out-of-range dispatch range have none), all in shared memory.
constexpr int TC_MAX_NE = 1024;
struct TileList {
  const int *pre, *cnt, *off;
  int NE;
};

// Calls f(e, m, pos0, nt) for this CTA's items: expert e, row tile m, tokens at dispatch positions [pos0, pos0 + nt).
// Every role of the CTA walks the same sequence. Stops (false) as soon as f fails.
template <int NT, class F>
CLB_DEV bool for_each_tile(const TileList &L, int MT, F &&f) {
  const int total = L.pre[L.NE];
  for (int w = blockIdx.x; w < total; w += gridDim.x) {
    int lo = 0, hi = L.NE - 1;   // the last expert whose items start at or before w (it has items: pre[e + 1] > w)
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (L.pre[mid] <= w) lo = mid;
      else hi = mid - 1;
    }
    const int e = lo, n_e = L.cnt[e], nch = (n_e + NT - 1) / NT, local = w - L.pre[e];
    const int m = local / nch, n0 = (local - m * nch) * NT;
    if (m >= MT || n0 >= n_e) continue;   // cannot happen for a consistent list
    if (!f(e, m, L.off[e] + n0, min(NT, n_e - n0))) return false;
  }
  return true;
}

}  // namespace

template <bool GATEUP, uint32_t WT>
__global__ void __launch_bounds__(TC_THREADS, 1)
    group_tc_kernel(const BatchArgs a, const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                    const __grid_constant__ CUtensorMap tm_bh, const __grid_constant__ CUtensorMap tm_bl) {
  using S = TcShape<WT>;
  constexpr int NT = S::NT, RAW_STAGES = S::RAW_STAGES, A_STAGES = S::A_STAGES, B_STAGES = S::B_STAGES;
  constexpr bool STACK = S::STACK;
  constexpr uint32_t RAW_STAGE = S::RAW_STAGE, B_STAGE = S::B_STAGE, ACC_COLS = S::ACC_COLS;
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

  __shared__ int s_pre[TC_MAX_NE + 1], s_cnt[TC_MAX_NE], s_off[TC_MAX_NE];
  {   // the work list: each expert's tokens (none for an out-of-range dispatch range), then the prefix of its items
    const int TK = a.T * a.K;
    for (int e = threadIdx.x; e < a.NE; e += blockDim.x) {
      const int n_e = a.counts[e], p0 = a.offsets[e];
      const bool good = n_e > 0 && p0 >= 0 && p0 + n_e <= TK;
      s_cnt[e] = good ? n_e : 0;
      s_off[e] = good ? p0 : 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int acc = 0;
      for (int e = 0; e < a.NE; ++e) {
        s_pre[e] = acc;
        acc += MT * ((s_cnt[e] + NT - 1) / NT);
      }
      s_pre[a.NE] = acc;
    }
  }
  const TileList tl{s_pre, s_cnt, s_off, a.NE};
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
      ok = for_each_tile<NT>(tl, MT, [&](int e, int m, int, int) {
        for (int c = 0; c < nchunk; ++c) {
          for (int mA = 0; mA < 2; ++mA, ++u) {
            const uint32_t s = u % RAW_STAGES;
            if (u >= RAW_STAGES && !mbar_wait_bounded(&raw_free[s], (u / RAW_STAGES - 1) & 1)) return false;
            const int y = e * rows_e + (GATEUP ? 128 * m : 256 * m + 128 * mA);
            mbar_arrive_expect_tx(&raw_full[s], RAW_STAGE);
            tma_load_2d(raw + s * RAW_STAGE, mA ? &tm_w1 : &tm_w0, static_cast<int>(S::CHUNK / 8) * c, y, &raw_full[s]);
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
      ok = for_each_tile<NT>(tl, MT, [&](int, int, int pos0, int nt) {
        const int NTt = (nt + 15) & ~15;
        for (int c = 0; c < nchunk; ++c) {
          for (int at = 0; at < 4; ++at, ++t) {
            const uint32_t s = t % B_STAGES;
            if (t >= B_STAGES && !mbar_wait_bounded(&b_free[s], (t / B_STAGES - 1) & 1)) return false;
            mbar_arrive_expect_tx(&b_full[s], static_cast<uint32_t>(NTt) * 256u);
            uint8_t *bs = bst + s * B_STAGE;
            for (int j = 0; j < NTt / 16; ++j) {
              tma_load_2d(bs + 2048 * j, &tm_bh, 256 * c + 64 * at, pos0 + 16 * j, &b_full[s]);
              tma_load_2d(bs + 128 * NTt + 2048 * j, &tm_bl, 256 * c + 64 * at, pos0 + 16 * j, &b_full[s]);
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
      const uint32_t acc = tmem + (STACK ? 2 : 1) * NT * mA;
      uint32_t t = 0, it = 0;
      ok = for_each_tile<NT>(tl, MT, [&](int, int, int, int nt) {
        const int NTt = (nt + 15) & ~15;
        const uint32_t idesc = tc::idesc_f16_f32(128, (STACK ? 2 : 1) * NTt);
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
            if constexpr (STACK) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {   // K step: +8 TMEM columns of A, +32 bytes (2 descriptor units) of B
                tc::mma_f16_ts(acc, ah + 8 * kk, bdesc + 2 * kk, idesc, c != 0 || at != 0 || kk != 0);
                tc::mma_f16_ts(acc, ah + 32 + 8 * kk, bdesc + 2 * kk, idesc, true);
              }
            } else {
              // x lo rows start 128 NTt bytes in: a multiple of 2048, so a fresh 128-byte-swizzle tile
              const uint64_t bdesc_lo = tc::sw128_desc(smem_addr(bst + sb * B_STAGE + 128 * NTt));
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                tc::mma_f16_ts(acc, ah + 8 * kk, bdesc + 2 * kk, idesc, c != 0 || at != 0 || kk != 0);   // w hi x hi
                tc::mma_f16_ts(acc, ah + 8 * kk, bdesc_lo + 2 * kk, idesc, true);                         // w hi x lo
                tc::mma_f16_ts(acc, ah + 32 + 8 * kk, bdesc + 2 * kk, idesc, true);                       // w lo x hi
              }
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
    ok = for_each_tile<NT>(tl, MT, [&](int, int m, int pos0, int nt) {
      for (int c = 0; c < nchunk; ++c, ++g) {
        const uint32_t u = 2 * g + mA, s = u % RAW_STAGES;
        if (!mbar_wait_bounded(&raw_full[s], (u / RAW_STAGES) & 1)) return false;
        // this thread's weight row of the chunk, read from the stage atom by atom (the stage is released after the last)
        const uint32_t *rw = reinterpret_cast<const uint32_t *>(raw + s * RAW_STAGE + r * S::CHUNK);
        uint32_t hdr[4] = {0, 0, 0, 0};
        if constexpr (WT != T_Q8_0) {
          const uint4 h4 = *reinterpret_cast<const uint4 *>(rw);
          hdr[0] = h4.x; hdr[1] = h4.y; hdr[2] = h4.z; hdr[3] = h4.w;
        }
#pragma unroll 1
        for (int at = 0; at < 4; ++at, ++t) {
          constexpr int AW = WT == T_Q8_0 ? 17 : 8;
          uint32_t aw[AW];
          if constexpr (WT == T_Q8_0) {
#pragma unroll
            for (int i = 0; i < 17; ++i) aw[i] = rw[17 * at + i];
          } else {
            const uint4 *p4 = reinterpret_cast<const uint4 *>(rw + 4 + 8 * at);
            const uint4 x0 = p4[0], x1 = p4[1];
            aw[0] = x0.x; aw[1] = x0.y; aw[2] = x0.z; aw[3] = x0.w; aw[4] = x1.x; aw[5] = x1.y; aw[6] = x1.z; aw[7] = x1.w;
          }
          const uint32_t sa = t % A_STAGES;
          if (t >= A_STAGES && !mbar_wait_bounded(&a_free[sa], (t / A_STAGES - 1) & 1)) return false;
          tc::fence_after_sync();
          const uint32_t col = tmem + lane_base + ACC_COLS + A_COLS * sa + 64 * mA;
#pragma unroll
          for (int bb = 0; bb < 2; ++bb) {   // two 32-element pieces: Q8_0 blocks, Q4_K sub-blocks
            uint32_t hi[16], lo[16];
            if constexpr (WT == T_Q8_0) dequant_q80_atom(aw, bb, hi, lo);
            else dequant_q4k_atom(hdr, aw, 2 * at + bb, hi, lo);
            tc::st_x16(col + 16 * bb, hi);
            tc::st_x16(col + 32 + 16 * bb, lo);
          }
          tc::wait_st();
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[sa]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_free[s]);
      }
      // epilogue: warps of matrix 0 take tokens [0, NT/2), those of matrix 1 [NT/2, NT), 16 at a time; each reads both
      // accumulators (STACK: column n holds the x hi products and column NTt + n the x lo products of token n)
      if (!mbar_wait_bounded(acc_full, it & 1)) return false;
      tc::fence_after_sync();
      const int NTt = (nt + 15) & ~15;
#pragma unroll 1
      for (int h = 0; h < NT / 32; ++h) {
        const int c0 = (NT / 2) * mA + 16 * h;
        if (c0 >= nt) break;   // warp-uniform
        float v0[16], v1[16];
        if constexpr (STACK) {
          float l0[16], l1[16];
          tc::ld_x16(tmem + lane_base + c0, v0);
          tc::ld_x16(tmem + lane_base + NTt + c0, l0);
          tc::ld_x16(tmem + lane_base + 2 * NT + c0, v1);
          tc::ld_x16(tmem + lane_base + 2 * NT + NTt + c0, l1);
#pragma unroll
          for (int j = 0; j < 16; ++j) { v0[j] = __fadd_rn(v0[j], l0[j]); v1[j] = __fadd_rn(v1[j], l1[j]); }
        } else {
          tc::ld_x16(tmem + lane_base + c0, v0);
          tc::ld_x16(tmem + lane_base + NT + c0, v1);
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int n = c0 + j;
          if (n >= nt) break;
          const size_t pos = static_cast<size_t>(pos0 + n);
          if constexpr (WT != T_Q8_0) {   // undo the planes' power-of-two row scale (exact)
            const float sc = a.rs[pos];
            v0[j] = __fmul_rn(v0[j], sc);
            v1[j] = __fmul_rn(v1[j], sc);
          }
          if (GATEUP) {
            const float hv = silu_mul_once(v0[j], v1[j]);
            const size_t o = pos * a.FF + 128 * m + r;
            a.hg[o] = hv;
            if (a.tc_dn && a.down_type == T_Q8_0) {   // the Q8_0 down product's activations
              const __half hh = __float2half_rn(hv);
              a.hgh[o] = hh;
              a.hgl[o] = __float2half_rn(__fsub_rn(hv, __half2float(hh)));
            }
          } else {
            const size_t o = pos * a.E + 256 * m + r;
            a.hd[o] = v0[j];
            a.hd[o + 128] = v1[j];
          }
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_free);
      ++it;
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

// Gathers the fp16 hi/lo planes of xn into dispatch order (row p = the token at dispatch position p). Q8_0 experts.
__global__ void gather_x_kernel(const BatchArgs a) {
  const int p = blockIdx.x;
  if (p >= a.offsets[a.NE]) return;   // not a dispatched slot
  const int t = a.pos_token[p];
  if (t < 0 || t >= a.T) { if (threadIdx.x == 0) set_error(a.err, ERR_BAD_EXPERT); return; }
  const uint4 *sh = reinterpret_cast<const uint4 *>(a.xh + static_cast<size_t>(t) * a.E);
  const uint4 *sl = reinterpret_cast<const uint4 *>(a.xl + static_cast<size_t>(t) * a.E);
  uint4 *dh = reinterpret_cast<uint4 *>(a.xdh + static_cast<size_t>(p) * a.E);
  uint4 *dl = reinterpret_cast<uint4 *>(a.xdl + static_cast<size_t>(p) * a.E);
  for (int i = threadIdx.x; i < a.E / 8; i += blockDim.x) { dh[i] = sh[i]; dl[i] = sl[i]; }
}

// The value of a Q8_K row (yd * q8 per 256-element block) as fp16 hi/lo planes, row p of the output, for p below *count
// (the dispatched slots). K-quant experts: gate/up read the token's Q8_K row of xn (row_of: the token at dispatch
// position p), down reads the Q8_K row of hg at position p itself (row_of null). The row is divided by rs[p] = 2^k, k the
// exponent of its largest block scale, so every value lies within +-254 whatever the row's range (hg rows can exceed
// fp16's); division by a power of two is exact, and the tensor-core epilogue multiplies rs[p] back.
__global__ void q8k_planes_kernel(const int8_t *qs, const float *d, int n, const int *row_of, int rows, const int *count, __half *outh,
                                  __half *outl, float *rs, int *err) {
  const int p = blockIdx.x;
  if (p >= *count) return;
  const int src = row_of ? row_of[p] : p;
  if (src < 0 || src >= rows) { if (threadIdx.x == 0) set_error(err, ERR_BAD_EXPERT); return; }
  const int8_t *q = qs + static_cast<size_t>(src) * n;
  const float *dd = d + static_cast<size_t>(src) * (n / 256);
  float mx = 0.f;
  for (int b = 0; b < n / 256; ++b) mx = fmaxf(mx, dd[b]);
  const float scale = mx > 0.f ? ldexpf(1.0f, ilogbf(mx)) : 1.0f;
  const float inv = 1.0f / scale;   // a power of two: exact
  if (threadIdx.x == 0) rs[p] = scale;
  for (int i = 2 * threadIdx.x; i < n; i += 2 * blockDim.x) {
    const float yd = __fmul_rn(dd[i / 256], inv);
    const float v0 = __fmul_rn(yd, static_cast<float>(q[i])), v1 = __fmul_rn(yd, static_cast<float>(q[i + 1]));
    const __half2 h = __floats2half2_rn(v0, v1);
    const __half2 l = __floats2half2_rn(__fsub_rn(v0, __low2float(h)), __fsub_rn(v1, __high2float(h)));
    reinterpret_cast<__half2 *>(outh + static_cast<size_t>(p) * n)[i / 2] = h;
    reinterpret_cast<__half2 *>(outl + static_cast<size_t>(p) * n)[i / 2] = l;
  }
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

// A 2-D map over weight rows [rows x row_bytes] (all experts' rows one after another), in 8-byte units: boxes of one
// 256-element chunk (`chunk` bytes) x 128 rows, no swizzle (rows land `chunk` bytes apart).
static bool encode_raw(CUtensorMap *m, const void *base, int rows, uint32_t row_bytes, uint32_t chunk) {
  const EncodeTiled fn = encoder();
  if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes % chunk) || (row_bytes % 16)) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes / 8), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  const cuuint32_t box[2] = {chunk / 8, 128}, estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tc_type_supported(uint32_t type, const void *w, int E, int FF) {
  return (type == T_Q8_0 || type == T_Q4_K) && (reinterpret_cast<uintptr_t>(w) & 15) == 0 && E % 256 == 0 && FF % 256 == 0 &&
         E >= 256 && FF >= 256;
}

template <bool GATEUP, uint32_t WT>
static int launch_kernel(const BatchArgs &a, cudaStream_t st, const CUtensorMap &tw0, const CUtensorMap &tw1, const CUtensorMap &tbh,
                         const CUtensorMap &tbl) {
  int dev = 0;
  cudaGetDevice(&dev);
  static int sms[64] = {};
  if (dev < 0 || dev >= 64) return static_cast<int>(cudaErrorInvalidDevice);
  if (!sms[dev]) {
    cudaFuncSetAttribute(group_tc_kernel<GATEUP, WT>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcShape<WT>::SMEM);
    cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  }
  const long chunks = (static_cast<long>(a.T) * a.K + TcShape<WT>::NT - 1) / TcShape<WT>::NT;   // an expert's at most
  const long items = static_cast<long>(a.NE) * (GATEUP ? a.FF / 128 : a.E / 256) * chunks;
  const int grid = items < sms[dev] ? static_cast<int>(items) : sms[dev];
  group_tc_kernel<GATEUP, WT><<<grid, TC_THREADS, TcShape<WT>::SMEM, st>>>(a, tw0, tw1, tbh, tbl);
  return static_cast<int>(cudaGetLastError());
}

int launch_tc(const BatchArgs &a, void *stream_, bool gateup) {
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  if (a.NE > TC_MAX_NE || a.NE < 1) return static_cast<int>(cudaErrorInvalidValue);
  const int TK = a.T * a.K;
  const uint32_t wt = gateup ? a.gate_type : a.down_type;
  const uint32_t chunk = wt == T_Q8_0 ? TcShape<T_Q8_0>::CHUNK : TcShape<T_Q4_K>::CHUNK;
  CUtensorMap tw0, tw1, tbh, tbl;
  bool ok;
  if (gateup) {
    if (wt == T_Q8_0) gather_x_kernel<<<TK, 256, 0, st>>>(a);
    else q8k_planes_kernel<<<TK, 256, 0, st>>>(a.xq_qs, a.xq_d, a.E, a.pos_token, a.T, a.offsets + a.NE, a.xdh, a.xdl, a.rs, a.err);
    ok = encode_raw(&tw0, a.gate, a.NE * a.FF, a.grb, chunk) && encode_raw(&tw1, a.up, a.NE * a.FF, a.grb, chunk) &&
         encode_plane(&tbh, a.xdh, TK, a.E) && encode_plane(&tbl, a.xdl, TK, a.E);
  } else {
    if (wt != T_Q8_0) q8k_planes_kernel<<<TK, 256, 0, st>>>(a.hq_qs, a.hq_d, a.FF, nullptr, TK, a.offsets + a.NE, a.hgh, a.hgl, a.rs, a.err);
    ok = encode_raw(&tw0, a.down, a.NE * a.E, a.drb, chunk) && encode_raw(&tw1, a.down, a.NE * a.E, a.drb, chunk) &&
         encode_plane(&tbh, a.hgh, TK, a.FF) && encode_plane(&tbl, a.hgl, TK, a.FF);
  }
  if (!ok) return static_cast<int>(cudaErrorInvalidValue);
  if (gateup) return wt == T_Q8_0 ? launch_kernel<true, T_Q8_0>(a, st, tw0, tw1, tbh, tbl) : launch_kernel<true, T_Q4_K>(a, st, tw0, tw1, tbh, tbl);
  return wt == T_Q8_0 ? launch_kernel<false, T_Q8_0>(a, st, tw0, tw1, tbh, tbl) : launch_kernel<false, T_Q4_K>(a, st, tw0, tw1, tbh, tbl);
}

// A dense Q4_K matrix (rows x cols, row stride rb) times nb tokens' plain Q8_K rows on the tensor cores: the grouped kernel
// with one "expert" holding every token (the down role: row tiles of 256, token chunks spread over the CTAs, the
// activations as fp16 hi/lo planes scaled by a power of two per token). co: device ints {nb, 0, nb} (the expert's count
// and offsets). out [nb][rows].
int launch_tc_dense(const uint8_t *w, uint32_t rb, int rows, int cols, int nb, const int8_t *qs, const float *dd, int *co,
                    __half *ph, __half *pl, float *rs, float *out, int *err, cudaStream_t st) {
  if (!tc_type_supported(T_Q4_K, w, rows, cols) || nb < 1) return static_cast<int>(cudaErrorInvalidValue);
  BatchArgs b{};
  b.T = nb;
  b.K = 1;
  b.NE = 1;
  b.E = rows;
  b.FF = cols;
  b.down = w;
  b.down_type = T_Q4_K;
  b.drb = rb;
  b.down_slab = static_cast<uint64_t>(rows) * rb;
  b.counts = co;
  b.offsets = co + 1;
  b.hq_qs = const_cast<int8_t *>(qs);
  b.hq_d = const_cast<float *>(dd);
  b.hgh = ph;
  b.hgl = pl;
  b.rs = rs;
  b.hd = out;
  b.err = err;
  b.tc_dn = 1;
  return launch_tc(b, st, false);
}

}  // namespace clb
