// Batched expert products on the 5th-generation tensor cores (tcgen05, accumulators in TMEM) for Q8_0 experts: the
// gate/up and down products of the reference's batched block (c/src/forward.c:1197-1201) as grouped GEMMs.
//
// A CTA takes one expert and 256 weight rows: gate rows [128m, 128m+128) and up rows of the same range (gate/up), or down
// rows [256m, 256m+256) (down); one thread per weight row. Per 256-element chunk of K each thread loads its row's 272
// bytes (8 Q8_0 blocks) into registers one chunk ahead, and per 64-element atom it writes the row's dequantized weights
// as two fp16 planes, hi = fp16(q*d) and lo = fp16(q*d - hi) (half2 arithmetic: exact products, one rounding each), into
// shared memory in the canonical 128-byte-swizzled K-major layout. The activations of the expert's tokens (dispatch
// order) come as fp16 hi/lo planes too. One thread issues, per 16-element K step and per weight matrix, three MMAs
// (hi*hi + hi*lo + lo*hi) into an fp32 TMEM accumulator of 128 rows x N tokens: products accurate to about 2^-22, so the
// result stays within 1e-6 relative of the reference's fp32 float path (c/src/quant.c:889-902) instead of the ~4e-4
// that single fp16 operands give. Two shared-memory stages let the dequantization of one atom overlap the MMAs of the
// previous one. Epilogue: gate/up -> SwiGLU -> hg as fp16 hi/lo planes (the down product's activations); down -> hd fp32.
#include <cuda.h>
#include <cuda_fp16.h>

#include <cstring>

#include "common.cuh"
#include "decode.cuh"
#include "tcgen05.cuh"

namespace clb {

namespace {

constexpr int TC_THREADS = 256;
constexpr int TC_NT = 32;                        // tokens per accumulator tile
constexpr uint32_t A_TILE = 128 * 128;           // 128 rows x 64 fp16
constexpr uint32_t A_STAGE = 4 * A_TILE;         // A0 hi, A0 lo, A1 hi, A1 lo
constexpr uint32_t B_TILE = TC_NT * 128;         // up to 32 tokens x 64 fp16
constexpr uint32_t B_STAGE = 2 * B_TILE;         // B hi, B lo
constexpr int A_STAGES = 2, B_STAGES = 4;
constexpr uint32_t SMEM_BYTES = A_STAGES * A_STAGE + B_STAGES * B_STAGE + 1024 + 128;

// 2-D tiled TMA load of one box (64 fp16 x 16 rows, 128-byte swizzle) into shared memory, completing on `bar`.
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

// Writes atom `at` (64 elements = Q8_0 blocks 2at and 2at+1 of the chunk) of this thread's row into the hi and lo tiles.
CLB_DEV void write_atom(const uint32_t (&w)[68], int at, uint8_t *hi_tile, uint8_t *lo_tile, int r) {
#pragma unroll
  for (int bb = 0; bb < 2; ++bb) {
    const int b = 2 * at + bb;
    const uint32_t dw = w[(34 * b) >> 2];   // the block's fp16 scale at byte 34b (2-byte aligned)
    const __half2 d2 = __half2half2(__ushort_as_half(static_cast<unsigned short>(((34 * b) & 3) == 0 ? (dw & 0xffffu) : (dw >> 16))));
#pragma unroll
    for (int c = 0; c < 4; ++c) {   // 8 values -> one 16-byte chunk of each plane
      const uint32_t q0 = word_at(w, 34 * b + 2 + 8 * c), q1 = word_at(w, 34 * b + 6 + 8 * c);
      uint4 hv, lv;
      dequant4(q0, d2, hv.x, hv.y, lv.x, lv.y);
      dequant4(q1, d2, hv.z, hv.w, lv.z, lv.w);
      const uint32_t off = tc::sw128_chunk(r, 4 * bb + c);
      *reinterpret_cast<uint4 *>(hi_tile + off) = hv;
      *reinterpret_cast<uint4 *>(lo_tile + off) = lv;
    }
  }
}

}  // namespace

template <bool GATEUP>
__global__ void __launch_bounds__(TC_THREADS, 1)
    q80_group_tc_kernel(const BatchArgs a, const __grid_constant__ CUtensorMap tm_hi, const __grid_constant__ CUtensorMap tm_lo) {
  const int e = blockIdx.x, n_e = a.counts[e];
  if (n_e == 0) return;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *astage = smem, *bstage = smem + A_STAGES * A_STAGE;
  uint64_t *afree = reinterpret_cast<uint64_t *>(bstage + B_STAGES * B_STAGE);   // [2] A stage free (its MMAs done)
  uint64_t *bfull = afree + 2;                                                      // [4] B stage landed (TMA)
  uint64_t *bfree = bfull + 4;                                                      // [4] B stage free
  uint64_t *done = bfree + 4;                                                       // [1] a token tile's MMAs done
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = GATEUP ? a.E : a.FF;                 // reduction length
  const uint32_t rb = static_cast<uint32_t>(K / 32 * 34);
  const int mA = tid >> 7, r = tid & 127;            // this thread's weight matrix (0/1) and row
  const int row_g = GATEUP ? 128 * blockIdx.y + r : 256 * blockIdx.y + 128 * mA + r;
  const uint8_t *wrow = GATEUP ? (mA == 0 ? a.gate : a.up) + static_cast<size_t>(e) * a.gate_slab + static_cast<size_t>(row_g) * rb
                               : a.down + static_cast<size_t>(e) * a.down_slab + static_cast<size_t>(row_g) * rb;
  const int p0 = a.offsets[e];
  if (p0 < 0 || p0 + n_e > a.T * a.K) { if (tid == 0) set_error(a.err, ERR_BAD_EXPERT); return; }
  const int nchunk = K / 256, per_tile = 4 * nchunk, ntiles = (n_e + TC_NT - 1) / TC_NT, total = ntiles * per_tile;

  if (tid == 0) {
    for (int i = 0; i < 11; ++i) mbar_init(&afree[i], 1);
    fence_barrier_init();
  }
  if (warp == 0) tc::tmem_alloc(tmem_slot, 64);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot, acc[2] = {tmem, tmem + 32};
  bool failed = false;

  // B (the tokens' activations, dispatch order) of atom i: rows p0 + 32*tile .. +NT, K columns 64*(i % per_tile) ..
  auto issue_b = [&](int i) {   // thread 0
    const int tile = i / per_tile, k0 = 64 * (i - tile * per_tile);
    const int NTt = (min(TC_NT, n_e - TC_NT * tile) + 15) & ~15;
    uint8_t *bs = bstage + (i & 3) * B_STAGE;
    mbar_arrive_expect_tx(&bfull[i & 3], static_cast<uint32_t>(NTt) * 256u);
    for (int j = 0; j < NTt / 16; ++j) {
      tma_load_2d(bs + 2048 * j, &tm_hi, k0, p0 + TC_NT * tile + 16 * j, &bfull[i & 3]);
      tma_load_2d(bs + B_TILE + 2048 * j, &tm_lo, k0, p0 + TC_NT * tile + 16 * j, &bfull[i & 3]);
    }
  };
  if (tid == 0) {
    issue_b(0);
    if (total > 1) issue_b(1);
  }

  int atom = 0;
  for (int tile = 0; tile < ntiles; ++tile) {
    const int nt0 = TC_NT * tile, nt = min(TC_NT, n_e - nt0), NT = (nt + 15) & ~15;
    const uint32_t idesc = tc::idesc_f16_f32(128, NT);
    uint32_t raw[68], nxt[68];
    {
      const uint4 *src = reinterpret_cast<const uint4 *>(wrow);
#pragma unroll
      for (int i = 0; i < 17; ++i) {
        const uint4 v = __ldcs(src + i);
        raw[4 * i] = v.x; raw[4 * i + 1] = v.y; raw[4 * i + 2] = v.z; raw[4 * i + 3] = v.w;
      }
    }
    for (int c = 0; c < nchunk; ++c) {
      if (c + 1 < nchunk) {
        const uint4 *src = reinterpret_cast<const uint4 *>(wrow + static_cast<size_t>(c + 1) * 272);
#pragma unroll
        for (int i = 0; i < 17; ++i) {
          const uint4 v = __ldcs(src + i);
          nxt[4 * i] = v.x; nxt[4 * i + 1] = v.y; nxt[4 * i + 2] = v.z; nxt[4 * i + 3] = v.w;
        }
      }
#pragma unroll
      for (int at = 0; at < 4; ++at, ++atom) {
        const int s = atom & 1, bs = atom & 3;
        if (tid == 0 && atom + 2 < total) {   // B two atoms ahead, once the MMAs that read its stage are done
          if (atom >= 2 && !mbar_wait_bounded(&bfree[(atom + 2) & 3], static_cast<uint32_t>(((atom - 2) >> 2) & 1))) failed = true;
          issue_b(atom + 2);
        }
        if (atom >= 2 && !mbar_wait_bounded(&afree[s], static_cast<uint32_t>(((atom >> 1) - 1) & 1))) failed = true;
        uint8_t *st = astage + s * A_STAGE;
        write_atom(raw, at, st + (2 * mA) * A_TILE, st + (2 * mA + 1) * A_TILE, r);
        fence_proxy_async();   // the A tiles were written by the generic proxy; the MMAs read them through the async proxy
        tc::fence_before_sync();
        __syncthreads();
        tc::fence_after_sync();
        if (tid == 0) {
          if (!mbar_wait_bounded(&bfull[bs], static_cast<uint32_t>((atom >> 2) & 1))) failed = true;
          tc::fence_after_sync();
          const uint32_t base = smem_addr(st);
          const uint32_t bh = smem_addr(bstage + bs * B_STAGE), bl = bh + B_TILE;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int m = 0; m < 2; ++m) {
              const uint32_t ah = base + (2 * m) * A_TILE, al = base + (2 * m + 1) * A_TILE;
              const bool first = (c == 0 && at == 0 && kk == 0);
              tc::mma_f16(acc[m], tc::sw128_desc(ah + 32 * kk), tc::sw128_desc(bh + 32 * kk), idesc, !first);
              tc::mma_f16(acc[m], tc::sw128_desc(ah + 32 * kk), tc::sw128_desc(bl + 32 * kk), idesc, true);
              tc::mma_f16(acc[m], tc::sw128_desc(al + 32 * kk), tc::sw128_desc(bh + 32 * kk), idesc, true);
            }
          }
          tc::commit(&afree[s]);
          tc::commit(&bfree[bs]);
        }
      }
#pragma unroll
      for (int i = 0; i < 68; ++i) raw[i] = nxt[i];
    }
    // epilogue: wait for this tile's MMAs, read the accumulators (warps 0-3: TMEM lanes = rows)
    if (tid == 0) tc::commit(done);
    if (!mbar_wait_bounded(done, static_cast<uint32_t>(tile & 1))) failed = true;
    tc::fence_after_sync();
    if (warp < 4) {
      const int row = 32 * warp + lane;
      const uint32_t lane_off = static_cast<uint32_t>(32 * warp) << 16;
      for (int c8 = 0; c8 < NT; c8 += 8) {
        float v0[8], v1[8];
        tc::ld_x8(acc[0] + lane_off + c8, v0);
        tc::ld_x8(acc[1] + lane_off + c8, v1);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int n = c8 + j;
          if (n >= nt) break;
          const int pos = p0 + nt0 + n;
          if (GATEUP) {
            const float h = silu_mul(v0[j], v1[j]);
            const __half hh = __float2half_rn(h);
            const __half hl = __float2half_rn(__fsub_rn(h, __half2float(hh)));
            const size_t o = static_cast<size_t>(pos) * a.FF + 128 * blockIdx.y + row;
            a.hgh[o] = hh;
            a.hgl[o] = hl;
          } else {
            const size_t o = static_cast<size_t>(pos) * a.E + 256 * blockIdx.y + row;
            a.hd[o] = v0[j];
            a.hd[o + 128] = v1[j];
          }
        }
      }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
  }
  if (failed) set_error(a.err, ERR_WAIT_COPY);
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 64);
}

template __global__ void q80_group_tc_kernel<true>(const BatchArgs, const __grid_constant__ CUtensorMap, const __grid_constant__ CUtensorMap);
template __global__ void q80_group_tc_kernel<false>(const BatchArgs, const __grid_constant__ CUtensorMap, const __grid_constant__ CUtensorMap);

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

// A 2-D fp16 tensor map over a [rows x cols] row-major plane: boxes of 64 columns x 16 rows, 128-byte swizzle (the
// canonical K-major layout the MMAs read), zeros outside the tensor.
static bool encode_plane(CUtensorMap *m, const void *base, int rows, int cols) {
  using Encode = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *, const cuuint64_t *,
                              const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static Encode fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess || !p) return false;
    fn = reinterpret_cast<Encode>(p);
  }
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {64, 16}, estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int launch_q80_tc(const BatchArgs &a, void *stream_, bool gateup) {
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  const int TK = a.T * a.K;
  CUtensorMap th, tl;
  if (gateup) {
    gather_x_kernel<<<TK, 256, 0, st>>>(a);
    if (!encode_plane(&th, a.xdh, TK, a.E) || !encode_plane(&tl, a.xdl, TK, a.E)) return static_cast<int>(cudaErrorInvalidValue);
  } else if (!encode_plane(&th, a.hgh, TK, a.FF) || !encode_plane(&tl, a.hgl, TK, a.FF)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attrs[64] = {};
  if (dev < 64 && !attrs[dev]) {
    cudaFuncSetAttribute(q80_group_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    cudaFuncSetAttribute(q80_group_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    attrs[dev] = true;
  }
  if (gateup) q80_group_tc_kernel<true><<<dim3(a.NE, a.FF / 128), TC_THREADS, SMEM_BYTES, st>>>(a, th, tl);
  else q80_group_tc_kernel<false><<<dim3(a.NE, a.E / 256), TC_THREADS, SMEM_BYTES, st>>>(a, th, tl);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace clb
