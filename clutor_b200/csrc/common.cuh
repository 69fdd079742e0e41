// Shared device code: PTX wrappers (mbarriers, bulk copies, programmatic dependent launch), bounded waits, and the
// exactly-rounded scalar steps of the reference's arithmetic.
//
// Parity rule for this whole library: the reference is built without FMA contraction (c/Makefile:3-9, -std=c11), so
// every float operation that must match it is written with an explicit round-to-nearest intrinsic (__fmul_rn, __fadd_rn,
// __fsub_rn, __fdiv_rn, __fsqrt_rn) and the library is compiled with --fmad=false.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#define CLB_DEV __device__ __forceinline__

namespace clb {

// ggml type ids (the reference's CL_T_*, c/src/quant.h:7)
constexpr uint32_t T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14;

// Device error codes written to the context's error word (first error wins).
enum : int { ERR_NONE = 0, ERR_WAIT_ROUTER = 1, ERR_WAIT_EXPERT = 2, ERR_WAIT_COPY = 3, ERR_BAD_EXPERT = 4, ERR_WAIT_GRID = 5,
             ERR_WAIT_PEER = 6 };

// A spin on a flag written by another CTA gives up after this many polls (each with a short sleep): about a second.
constexpr uint32_t SPIN_LIMIT = 1u << 22;

CLB_DEV uint32_t smem_addr(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// ---- mbarrier + bulk copy (global -> shared, this CTA only) -------------------------------------------------------------
CLB_DEV void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
CLB_DEV void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
CLB_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
CLB_DEV void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
CLB_DEV void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
// Untiled bulk copy: dst (shared) and src (global) 16-byte aligned, bytes a multiple of 16.
CLB_DEV void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}
// The same copy with an L2 cache policy (createpolicy): for data read once, evict-first keeps it from displacing what
// is read again (code, activations, caches).
CLB_DEV uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
CLB_DEV void bulk_copy_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t policy) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
               ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
               : "memory");
}
CLB_DEV bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for an mbarrier phase; false when the limit ran out.
CLB_DEV bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
#pragma unroll 1
  for (uint32_t i = 0; i < SPIN_LIMIT; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i > 64) __nanosleep(32);
  }
  return false;
}

// ---- programmatic dependent launch ---------------------------------------------------------------------------------------
CLB_DEV void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
CLB_DEV void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- inter-CTA flags -------------------------------------------------------------------------------------------------------
CLB_DEV uint32_t ld_acquire(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
CLB_DEV void red_release_add(uint32_t *p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Waits until *p >= target, for at most `limit` polls (about a second at SPIN_LIMIT). Call from one thread.
CLB_DEV bool wait_counter(const uint32_t *p, uint32_t target, uint32_t limit = SPIN_LIMIT) {
#pragma unroll 1
  for (uint32_t i = 0; i < limit; ++i) {
    if (ld_acquire(p) >= target) return true;
    if (i > 4096) __nanosleep(64);   // poll flat out for the first few microseconds: these waits are on the critical path
  }
  return false;
}
CLB_DEV void set_error(int *err, int code) { atomicCAS(err, 0, code); }

// ---- self-tagged words: a 32-bit value and the tag of the launch that wrote it, stored and loaded as one 64-bit word, so
// a reader that sees the tag it expects holds the value too (no separate flag, no ordering between two stores) ----------
CLB_DEV void st_word(unsigned long long *p, uint32_t tag, uint32_t bits) {
  const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | bits;
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
CLB_DEV unsigned long long ld_word(const unsigned long long *p) {
  unsigned long long w;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
// Waits (bounded) until the word at p carries `tag`; returns false when the limit ran out. *bits receives the value.
CLB_DEV bool wait_word(const unsigned long long *p, uint32_t tag, uint32_t *bits) {
#pragma unroll 1
  for (uint32_t i = 0; i < SPIN_LIMIT; ++i) {
    const unsigned long long w = ld_word(p);
    if (static_cast<uint32_t>(w >> 32) == tag) { *bits = static_cast<uint32_t>(w); return true; }
    if (i > 4096) __nanosleep(64);
  }
  return false;
}
CLB_DEV uint32_t ld_relaxed(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Acquire-release add; returns the old value.
CLB_DEV uint32_t atom_add_acq_rel(uint32_t *p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// ---- phase trace -------------------------------------------------------------------------------------------------------------
CLB_DEV unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t)::"memory");   // not moved across memory operations
  return t;
}
// Thread 0 of the CTA stamps boundary i of its row (32 entries per CTA) when tracing is on; trace_stamp_here stamps from
// whichever thread calls it. Boundaries hold the SM's cycle counter (exact within a CTA); entries 30 and 31 the global
// nanosecond timer at entry and exit (comparable across CTAs and launches).
constexpr int TRACE_ROW = 32;
CLB_DEV unsigned long long sm_cycles() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %clock64;" : "=l"(t)::"memory");
  return t;
}
CLB_DEV void trace_stamp_here(unsigned long long *trace, int i) {
  if (trace) trace[TRACE_ROW * blockIdx.x + i] = sm_cycles();
}
CLB_DEV void trace_time(unsigned long long *trace, int i) {
  if (trace && threadIdx.x == 0) trace[TRACE_ROW * blockIdx.x + i] = global_ns();
}
CLB_DEV void trace_stamp(unsigned long long *trace, int i) {
  if (threadIdx.x == 0) trace_stamp_here(trace, i);
}

// ---- packed fp32 (sm_100) ------------------------------------------------------------------------------------------------
// Two fp32 lanes per instruction (sm_100): each lane rounded once, as the scalar operation. There is deliberately no packed
// multiply: measured on the device, a packed multiply whose only use is a packed add came out fused (the router's dotf
// chains lost their bits), so products whose rounding matters stay scalar.
CLB_DEV unsigned long long f2_pack(float2 v) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(v.x), "f"(v.y));
  return r;
}
CLB_DEV float2 f2_unpack(unsigned long long r) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
CLB_DEV float2 ffma2(float2 a, float2 b, float2 c) {   // a * b + c
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(f2_pack(a)), "l"(f2_pack(b)), "l"(f2_pack(c)));
  return f2_unpack(r);
}
CLB_DEV float2 fadd2(float2 a, float2 b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_pack(a)), "l"(f2_pack(b)));
  return f2_unpack(r);
}
CLB_DEV float2 fsub2(float2 a, float2 b) {
  unsigned long long r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_pack(a)), "l"(f2_pack(b)));
  return f2_unpack(r);
}

// ---- the reference's scalar steps, exactly rounded ---------------------------------------------------------------------------
// fp16 bits to float: exact (every half is a float).
CLB_DEV float f16_bits_to_f32(uint16_t h) {
  float f;
  asm("{ .reg .b16 t; mov.b16 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "h"(h));
  return f;
}
// expf, correctly rounded except in vanishingly rare double-rounding cases: exp in double precision, rounded once to float.
// (The reference calls glibc's expf, which is within about half an ulp, so the two agree to an ulp.)
CLB_DEV float expf_cr(float x) { return __double2float_rn(exp(static_cast<double>(x))); }
// silu(g) * u as the reference writes it: g / (1 + expf(-g)) * u (c/src/forward.c:1018)
CLB_DEV float silu_mul(float g, float u) { return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf_cr(-g))), u); }

// Unaligned little-endian 32-bit load from shared memory (reads the aligned word after p too: keep 4 bytes of slack).
CLB_DEV uint32_t lds_u32_unaligned(const uint8_t *p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t *q = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
  return __funnelshift_r(q[0], q[1], static_cast<uint32_t>(a & 3) * 8u);
}
CLB_DEV uint16_t lds_u16(const uint8_t *p) { return static_cast<uint16_t>(p[0] | (p[1] << 8)); }

// 6-bit scale and min of sub-block j (0..7) of a Q4_K block from its 12 packed bytes (ggml layout; c/src/quant.c:36-40).
CLB_DEV void q4k_scale_min(const uint8_t *s12, int j, int &sc, int &mn) {
  if (j < 4) {
    sc = s12[j] & 63;
    mn = s12[j + 4] & 63;
  } else {
    sc = (s12[j + 4] & 15) | ((s12[j - 4] >> 6) << 4);
    mn = (s12[j + 4] >> 4) | ((s12[j] >> 6) << 4);
  }
}

CLB_DEV uint32_t block_elems(uint32_t t) { return t == T_Q8_0 ? 32u : 256u; }
CLB_DEV uint32_t block_bytes(uint32_t t) { return t == T_Q8_0 ? 34u : t == T_Q4_K ? 144u : 210u; }

}  // namespace clb
