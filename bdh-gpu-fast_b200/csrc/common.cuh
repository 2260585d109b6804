// Device-side primitives shared by every sm_100a kernel of the tril-attention path:
// mbarriers with bounded waits, TMA tile loads, tcgen05 (TMEM alloc, UMMA issue, commit,
// TMEM loads) and the shared-memory / instruction descriptors they consume.
//
// Every spin-wait in this library goes through `wait_bounded`: after BDH_WAIT_TIMEOUT_NS of
// wall time (read from %globaltimer) it records an error code in the caller-provided error
// word and returns false, so a broken pipeline ends the kernel instead of hanging the GPU.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#ifndef BDH_WAIT_TIMEOUT_NS
#define BDH_WAIT_TIMEOUT_NS 2000000000ull  // 2 s: far above any legitimate stage wait
#endif

namespace bdh {

// Error codes written to the device error word (host reads it after the launch).
enum : int {
  kErrNone = 0,
  kErrTimeoutProducer = 1,   // TMA producer gave up waiting for a free stage
  kErrTimeoutMma = 2,        // MMA issuer gave up waiting for a full stage / free accumulator
  kErrTimeoutEpilogue = 3,   // epilogue gave up waiting for a finished accumulator
  kErrTimeoutDrain = 4,      // teardown gave up waiting for in-flight MMAs
  kErrTimeoutDecode = 5,     // decode split reduction gave up waiting for peer splits
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t lane_id() {
  uint32_t l;
  asm volatile("mov.u32 %0, %laneid;" : "=r"(l));
  return l;
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 r;\n\t"
      "elect.sync r|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------- mbarrier ----
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for `bar` to complete the phase with the given parity. Gives up (returns false)
// when another role has raised `abort_flag` or after BDH_WAIT_TIMEOUT_NS; in the timeout
// case it raises the abort flag itself and records `code` in `err` (first error wins).
__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t parity,
                                             volatile int* abort_flag, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0u) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > BDH_WAIT_TIMEOUT_NS) {
        *abort_flag = 1;
        if (err != nullptr) atomicCAS(err, 0, code);
        return false;
      }
    }
  }
}

// --------------------------------------------------------------------- TMA ----
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 4-D tiled load (coordinates innermost first) completing on `bar` with byte accounting.
__device__ __forceinline__ void tma_load_4d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}

// L2 cache policies for TMA copies: operands that many tiles re-read stay (evict_last);
// streams that are read or written once go first (evict_first).
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// 16-byte global store with an L2 cache policy.
__device__ __forceinline__ void st_global_v4_hint(void* p, uint4 v, uint64_t policy) {
  asm volatile("st.global.L2::cache_hint.v4.b32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w), "l"(policy)
               : "memory");
}

// Transpose of an 8 x 8 matrix of 16-byte chunks inside each group of 8 lanes of a warp
// (three exchange stages of 4 chunks with the lane at distance 4, 2, 1). On entry lane i of a
// group holds row i (c[k] = element (i, k)); on exit lane j holds column j (c[k] = element (k, j)).
// A thread that owns one tile row can then store 8 consecutive chunks of one row per group:
// 128 contiguous bytes per 8 lanes instead of 32 rows per warp instruction.
__device__ __forceinline__ void transpose_chunks8(uint4 (&c)[8], int lane) {
#pragma unroll
  for (int m = 4; m >= 1; m >>= 1) {
    const bool hi = (lane & m) != 0;
#pragma unroll
    for (int k0 = 0; k0 < 8; ++k0) {
      if (k0 & m) continue;
      const int k1 = k0 | m;
      const uint4 s = hi ? c[k0] : c[k1];
      uint4 r;
      r.x = __shfl_xor_sync(0xffffffffu, s.x, m);
      r.y = __shfl_xor_sync(0xffffffffu, s.y, m);
      r.z = __shfl_xor_sync(0xffffffffu, s.z, m);
      r.w = __shfl_xor_sync(0xffffffffu, s.w, m);
      if (hi)
        c[k0] = r;
      else
        c[k1] = r;
    }
  }
}

__device__ __forceinline__ void tma_load_4d_hint(const CUtensorMap* map, uint64_t* bar, void* dst,
                                                 int c0, int c1, int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_store_4d_hint(const CUtensorMap* map, const void* src, int c0,
                                                  int c1, int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group.L2::cache_hint"
      " [%0, {%2, %3, %4, %5}], [%1], %6;"
      ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3), "l"(policy)
      : "memory");
}

// 4-D tiled store from shared memory (bulk-group completion). The source must be visible to
// the async proxy: every writing thread executes fence_async_smem() before the issuing thread
// is released.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0,
                                             int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];"
      ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until every committed bulk store has finished READING its shared-memory source.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until every committed bulk store has completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------------- tcgen05 ----
// Allocate `ncols` TMEM columns (power of two >= 32); executed by one full warp.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Programmatic dependent launch. A kernel launched with programmatic stream serialization may
// begin while the previous kernel of its stream still runs; pdl_wait() returns once that kernel
// has completed and its writes are visible (immediately for a kernel launched without the
// attribute), so every thread calls it before its first global-memory access, read or write.
// pdl_trigger() lets the stream's next such kernel begin launching its CTAs; that kernel still
// waits for this one's completion before touching memory.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16/fp16 operands, fp32 accumulate).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same with kind::tf32 (32-bit operands, the tensor core reads the tf32 part of each).
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Each thread of the warp reads 32 consecutive 32-bit columns of its own TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

// The same for 16 consecutive columns (32 lanes x 16 x 32-bit).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a 128-byte-swizzled operand tile.
//   K-major : rows of 128 B (one swizzle row), 8-row groups `sbo` bytes apart; LBO unused.
//   MN-major: 128-byte MN chunks `lbo` bytes apart, 8-row K groups `sbo` bytes apart.
// Bits: [0,14) addr>>4, [16,30) lbo>>4, [32,46) sbo>>4, [46,48) version 1,
//       [49,52) base offset 0, [61,64) layout 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// Instruction descriptor: fp32 accumulator, operand format `fmt` (1 = bf16 under kind::f16,
// 2 = tf32 under kind::tf32), majors (0 = K-major, 1 = MN-major), tile M x N.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t fmt, uint32_t a_mn, uint32_t b_mn,
                                                  uint32_t M, uint32_t N) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (a_mn << 15) | (b_mn << 16) |
         ((N >> 3) << 17) | ((M >> 4) << 24);
}

// ------------------------------------------------------------- conversions ----
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t bits16) {
  return __uint_as_float(bits16 << 16);
}

// Round-to-nearest-even bf16 of x, returned as the 16 raw bits. Integer arithmetic on the ALU
// pipes (the F2F conversion instruction issues on the 16-lane/clk XU pipe, which became the
// bottleneck of the RoPE pass); NaN inputs stay (quiet) NaN.
__device__ __forceinline__ uint32_t f32_to_bf16_bits(float x) {
  const uint32_t u = __float_as_uint(x);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (u >> 16) | 0x40u;
  return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}

// Two fp32 values to a packed bf16x2 word (lo in bits 0-15), round-to-nearest-even, with one
// conversion instruction for the pair.
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// relu then round, packed: {lo, hi} = {bf16(max(lo, 0)), bf16(max(hi, 0))} (NaN stays NaN).
__device__ __forceinline__ uint32_t cvt_relu_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.relu.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// Packed bf16 add / multiply, each the exact result rounded once to bf16 (round to nearest
// even): the same values as forming the sum / product in fp32 and rounding that, because the
// sum or product of two bf16 values needs at most 18 significant bits before the final
// rounding (fp32 then bf16 rounds innocuously, 24 >= 2 x 8 + 2).
__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ float bf16x2_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16x2_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// x rounded to the nearest bf16 value (ties to even), kept as fp32.
__device__ __forceinline__ float bf16_round_f32(float x) {
  return __uint_as_float(f32_to_bf16_bits(x) << 16);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) { return cvt_bf16x2(lo, hi); }


// ------------------------------------------------------------- fast division ----
// Division of 0 <= n < 2^31 by a divisor fixed at launch: q = umulhi(n, m) >> s with
// m = ceil(2^(31 + ceil(log2 d)) / d) (Granlund & Montgomery, "Division by invariant integers
// using multiplication", 1994), a multiply-high and a shift instead of the ~20-instruction
// integer division, for tile-index arithmetic on the issue paths of persistent kernels.
struct FastDiv {
  uint32_t d = 1, m = 0, s = 0;
  FastDiv() = default;
  __host__ explicit FastDiv(uint32_t divisor) : d(divisor) {
    if (d <= 1) return;  // m = 0 marks the identity
    uint32_t l = 0;
    while ((1ull << l) < d) ++l;  // ceil(log2 d)
    const uint64_t p = 31 + l;
    m = static_cast<uint32_t>(((1ull << p) + d - 1) / d);
    s = static_cast<uint32_t>(p - 32);
  }
  __device__ __forceinline__ int div(int n) const {
    if (m == 0) return n;
    return static_cast<int>(__umulhi(static_cast<uint32_t>(n), m) >> s);
  }
  __device__ __forceinline__ void divmod(int n, int& q, int& r) const {
    q = div(n);
    r = n - q * static_cast<int>(d);
  }
};

// ----------------------------------------------------------------- BDH RoPE ----
// cos / sin of the reference phase for position `pos` and frequency `f` (bdh.py:119-122,
// 142-150): fp32 product, exact fractional part (the product is >= 0), times fp32 2*pi as
// torch rounds the Python scalar (0x40C90FDB), then sincosf.
// (cos, sin) of the same phase with the hardware approximations (__sincosf) after reducing the
// phase to [-pi, pi), where their absolute error is below 2^-21. For gradients only (the RoPE
// adjoint of the backward): the forward rotation keeps rope_cis, whose values match the
// reference's fp32 cos / sin of the phase.
__device__ __forceinline__ void rope_cis_grad(float pos, float f, float& c, float& s) {
  float ph = __fmul_rn(pos, f);
  ph = __fsub_rn(ph, floorf(ph));
  if (ph >= 0.5f) ph -= 1.0f;
  __sincosf(__fmul_rn(ph, __int_as_float(0x40C90FDB)), &s, &c);
}
__device__ __forceinline__ void rope_cis(float pos, float f, float& c, float& s) {
  float ph = __fmul_rn(pos, f);
  ph = __fsub_rn(ph, floorf(ph));
  ph = __fmul_rn(ph, __int_as_float(0x40C90FDB));
  sincosf(ph, &s, &c);
}

// bf16 pair rotation (kernels/rope.py:108-126 with bf16 values and fp32 cos/sin): the four
// products are rounded to bf16 two at a time and the two bf16 sums rounded once more into the
// packed output word (y0 in the low half, y1 in the high half).
__device__ __forceinline__ uint32_t rotate_pair_bf16x2(float x0, float x1, float c0, float s0,
                                                       float c1, float s1) {
  const uint32_t a = cvt_bf16x2(__fmul_rn(x0, c0), __fmul_rn(x1, c1));   // x0 c0 | x1 c1
  const uint32_t b = cvt_bf16x2(__fmul_rn(-x1, s0), __fmul_rn(x0, s1));  // -x1 s0 | x0 s1
  return add_bf16x2(a, b);
}

}  // namespace bdh
