// Shared device helpers for the asterq kernels (sm_100a only).
//
// Everything here is either a thin inline-PTX wrapper around one instruction
// (mma.sync, ldmatrix, cp.async, packed f32x2 arithmetic) or plain integer /
// IEEE arithmetic.  No CUDA math-library internals are restated.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "asterq kernels are written for sm_100a (B200) only"
#endif

#define ASTERQ_DEVICE __device__ __forceinline__

namespace asterq {

// ---------------------------------------------------------------------------
// Packed float32x2 arithmetic (Blackwell add/sub/mul .f32x2).  Each lane of the
// pair is an ordinary IEEE round-to-nearest float32 operation, so results are
// bit-identical to two scalar operations.
// ---------------------------------------------------------------------------
ASTERQ_DEVICE unsigned long long f2_bits(float2 v) {
  return (unsigned long long)__float_as_uint(v.x) | ((unsigned long long)__float_as_uint(v.y) << 32);
}
ASTERQ_DEVICE float2 bits_f2(unsigned long long b) {
  return make_float2(__uint_as_float((unsigned)(b & 0xffffffffull)), __uint_as_float((unsigned)(b >> 32)));
}
ASTERQ_DEVICE float2 add2(float2 a, float2 b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}
ASTERQ_DEVICE float2 sub2(float2 a, float2 b) {
  unsigned long long d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}
ASTERQ_DEVICE float2 fma2(float2 a, float2 b, float2 c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
  return bits_f2(d);
}
ASTERQ_DEVICE float2 mul2(float2 a, float2 b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}

// ---------------------------------------------------------------------------
// bf16 / fp16 bit helpers
// ---------------------------------------------------------------------------
ASTERQ_DEVICE float bf16lo_to_f32(uint32_t w) { return __uint_as_float(w << 16); }
ASTERQ_DEVICE float bf16hi_to_f32(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

ASTERQ_DEVICE uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
ASTERQ_DEVICE uint32_t pack_bf162(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
ASTERQ_DEVICE float2 unpack_half2(uint32_t w) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  return __half22float2(h);
}
ASTERQ_DEVICE float2 unpack_bf162(uint32_t w) { return make_float2(bf16lo_to_f32(w), bf16hi_to_f32(w)); }

// fp16x2 arithmetic on raw 32-bit registers
ASTERQ_DEVICE uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
ASTERQ_DEVICE uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
ASTERQ_DEVICE uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
ASTERQ_DEVICE uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
// (a & mask) | bits, one LOP3
ASTERQ_DEVICE uint32_t and_or(uint32_t a, uint32_t mask, uint32_t bits) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(bits));
  return d;
}

// ---------------------------------------------------------------------------
// INT4 nibble -> fp16 conversion with the exponent-bias trick (published as the
// "magic number" int->float conversion, e.g. Kim et al. 2022, "Who Says
// Elephants Can't Run").  fp16 0x6400 is 1024.0 with an ulp of 1, so OR-ing a
// nibble u into its low mantissa bits gives exactly 1024 + u; a nibble sitting in
// mantissa bits 4..7 gives 1024 + 16u.  Codes are u - 8 in [-8, 7], exact in fp16.
// ---------------------------------------------------------------------------
constexpr uint32_t kF16Magic = 0x64006400u;   // (1024, 1024)
constexpr uint32_t kF16Bias1032 = 0x64086408u; // (1032, 1032)
constexpr uint32_t kF16Sixteenth = 0x2C002C00u; // (1/16, 1/16)
constexpr uint32_t kF16Minus72 = 0xD480D480u;  // (-72, -72)

// fp16x2 codes of the low nibbles at bit 0 and bit 16 of x
ASTERQ_DEVICE uint32_t nib_lo_f16x2(uint32_t x) { return hsub2_u32(and_or(x, 0x000F000Fu, kF16Magic), kF16Bias1032); }
// fp16x2 codes of the nibbles at bits 4..7 and 20..23 of x
ASTERQ_DEVICE uint32_t nib_hi_f16x2(uint32_t x) {
  return hfma2_u32(and_or(x, 0x00F000F0u, kF16Magic), kF16Sixteenth, kF16Minus72);
}

// float -> float8 e4m3 byte as torch's x.to(torch.float8_e4m3fn) writes it: the hardware
// conversion (round to nearest even, subnormals kept; it saturates 448 < |x| <= 464 to 448,
// where rounding to nearest even lands anyway), with NaN, infinities and |x| > 464 mapped to
// NaN carrying the sign of x
ASTERQ_DEVICE uint32_t f32_to_e4m3(float x) {
  unsigned short d;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %1;" : "=h"(d) : "f"(x));
  uint32_t code = d & 0xFFu;
  if (!(fabsf(x) <= 464.0f)) code = (__float_as_uint(x) >> 31) ? 0xFFu : 0x7Fu;
  return code;
}
// two e4m3 bytes (bits 0-7 and 8-15 of x) -> fp16x2, the low byte in the low half (exact:
// every e4m3 value is an fp16 value)
ASTERQ_DEVICE uint32_t e4m3x2_to_f16x2(uint32_t x) {
  uint32_t d;
  asm("{\n .reg .b16 t;\n cvt.u16.u32 t, %1;\n cvt.rn.f16x2.e4m3x2 %0, t;\n}" : "=r"(d) : "r"(x));
  return d;
}

// Signed bytes with the same trick: a byte v with its sign bit flipped is u = v + 128 in
// [0, 255], and 0x6400 | u is 1024 + u, so (x & 0x00FF00FF) ^ 0x64806480 (one LOP3) holds
// 1152 + v in each half and subtracting 1152 leaves v exactly.
constexpr uint32_t kF16Bias1152 = 0x64806480u;  // (1152, 1152), also the XOR pattern
ASTERQ_DEVICE uint32_t s8_bytes02_f16x2(uint32_t x) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(x), "r"(0x00FF00FFu), "r"(kF16Bias1152));  // (a & b) ^ c
  return hsub2_u32(d, kF16Bias1152);
}

// ---------------------------------------------------------------------------
// Warp-level tensor-core MMA (m16n8k16, fp32 accumulate)
// ---------------------------------------------------------------------------
// Register-only operations: not volatile, so the compiler may interleave
// independent MMAs to hide their latency.
ASTERQ_DEVICE void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
ASTERQ_DEVICE void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// int8 tensor path (m16n8k32, int32 accumulate).  mma_s8 accumulates in place;
// mma_s8_from starts every accumulator element at `c`.
ASTERQ_DEVICE void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
ASTERQ_DEVICE void mma_s8_from(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int c) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c));
}

// INT4 nibbles u = code + 8 -> signed bytes 16 * code: a nibble placed in the high half
// of a byte is 16u, and flipping bit 7 subtracts 128 = 16 * 8.  The four high nibbles
// (odd values of a packed word) need one logic op, the four low nibbles a shift first.
ASTERQ_DEVICE uint32_t s8_hi_nibbles(uint32_t x) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(x), "r"(0xF0F0F0F0u), "r"(0x80808080u));  // (a & b) ^ c
  return d;
}
ASTERQ_DEVICE uint32_t s8_lo_nibbles(uint32_t x) { return s8_hi_nibbles(x << 4); }

ASTERQ_DEVICE uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// 2^x by the hardware approximation with subnormal results flushed to zero (PTX
// ex2.approx.ftz.f32): softmax weights exp(s - max) <= 1, where a weight below 2^-126 is
// as good as zero
ASTERQ_DEVICE float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

ASTERQ_DEVICE void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}
ASTERQ_DEVICE void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

// ---------------------------------------------------------------------------
// Asynchronous global -> shared copies (16 bytes per thread, L2 only)
// ---------------------------------------------------------------------------
ASTERQ_DEVICE void cp_async16(uint32_t smem_addr, const void* gptr) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_addr), "l"(gptr));
}
ASTERQ_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
ASTERQ_DEVICE void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// ---------------------------------------------------------------------------
// mbarrier and bulk (TMA) copy helpers
// ---------------------------------------------------------------------------
ASTERQ_DEVICE void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
// an initialized mbarrier is invalidated before its slot is initialized again
ASTERQ_DEVICE void mbar_inval(uint32_t bar) {
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
ASTERQ_DEVICE void mbar_expect_tx(uint32_t bar, uint32_t tx) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(tx) : "memory");
}
ASTERQ_DEVICE void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
ASTERQ_DEVICE uint32_t mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok;
}
// try_wait that lets the hardware suspend the thread for up to `hint_ns`
// nanoseconds until the phase completes (it wakes as soon as it does), so a
// waiting warp takes almost no issue slots from the warps doing the work.
ASTERQ_DEVICE uint32_t mbar_try_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok;
}
ASTERQ_DEVICE int ld_shared_volatile(const volatile int* p) {
  int v;
  asm volatile("ld.volatile.shared.u32 %0, [%1];" : "=r"(v) : "r"((uint32_t)__cvta_generic_to_shared((const void*)p)) : "memory");
  return v;
}
// Bounded wait (`limit` SM clock cycles, by default 4e9: about 2 s): on timeout raise
// the CTA abort flag so every other wait returns at once and the kernel drains
// instead of hanging.  `abort_flag` points to shared memory.
constexpr long long kDefaultWaitLimit = 4000000000LL;
ASTERQ_DEVICE bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                             long long limit = kDefaultWaitLimit) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_sleep(bar, parity, 20000u)) return true;
    if (ld_shared_volatile(abort_flag)) return false;
    if (clock64() - t0 > limit) {
      *abort_flag = 1;
      return false;
    }
  }
}
ASTERQ_DEVICE void bulk_1d(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
ASTERQ_DEVICE void named_sync(int id, int count) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory"); }
ASTERQ_DEVICE void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }


ASTERQ_DEVICE uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

}  // namespace asterq
