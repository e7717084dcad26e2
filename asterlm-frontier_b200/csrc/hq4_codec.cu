// Cache write path (rotate -> groupwise absmax quantize -> nibble pack), its
// inverse, and the plain normalized FWHT.
//
// Reference algorithm (AsterLM-Frontier, src/asterlm/quantization/kv.py):
//   normalized_fwht  kv.py:13-32   butterflies h = 1, 2, ..., n/2, then / sqrt(n)
//   quantize_tensor  kv.py:76-118  scale = max(amax|g|, 1e-8) / qmax (fp32),
//                                  q = round_half_even(g / scale), clamp, pack
//   _pack_int4       kv.py:41-48   byte k = (q[2k]+8) | (q[2k+1]+8) << 4
//   dequantize_tensor kv.py:121-134
//
// All three kernels reproduce the reference bit for bit: every butterfly output
// is the same single IEEE float32 add/subtract of the same two operands, every
// division is correctly rounded, rounding is half-to-even.
//
// Register layout.  A token of D (padded, power-of-two) values is owned by
// LPT = D / EPL lanes of one warp, each holding EPL <= 128 consecutive values.
// Butterfly stages on the low log2(EPL) index bits run inside a lane; each of the
// remaining log2(LPT) stages pairs two lanes, which swap half of their values
// (one shuffle per pair of values) so that each lane can finish half of the
// butterflies locally.  After the last stage every lane owns runs of EPL/2
// consecutive values, so a quantization group (<= 64 values) never straddles
// lanes: absmax, rounding and nibble packing are lane-local.
#include "common.cuh"
#include "asterq_internal.h"

namespace asterq {

// x / c by the residual-correction step of Markstein (IBM J. Res. Dev. 34(1),
// 1990): q0 = x * r with r = RN(1/c), e = x - q0 * c (exact through the FMA),
// q1 = q0 + e * r.  For 2^-100 <= |x| <= 2^120 this is the correctly rounded
// quotient; tests/div_check.c verifies that over every float32 x for the two
// non-power-of-two divisors used here (sqrt(128), sqrt(512)) and over random
// (x, c) pairs in the quantizer's range.
ASTERQ_DEVICE float div_markstein(float x, float c, float r) {
  const float q0 = x * r;
  const float e = fmaf(-q0, c, x);
  return fmaf(e, r, q0);
}

// Correctly rounded x / c for every x: magnitudes outside Markstein's exact
// range (and NaN) take the IEEE division.
ASTERQ_DEVICE float div_by_const(float x, float c, float r) {
  const float ax = fabsf(x);
  if (ax >= 0x1p-100f && ax <= 0x1p120f) return div_markstein(x, c, r);
  return __fdiv_rn(x, c);
}

template <int EPL>
ASTERQ_DEVICE void fwht_local(float (&v)[EPL]) {
  // stage h = 1: pairs (2k, 2k+1)
#pragma unroll
  for (int k = 0; k < EPL; k += 2) {
    float a = v[k], b = v[k + 1];
    v[k] = a + b;
    v[k + 1] = a - b;
  }
#pragma unroll
  for (int h = 2; h < EPL; h *= 2) {
#pragma unroll
    for (int blk = 0; blk < EPL; blk += 2 * h) {
#pragma unroll
      for (int j = 0; j < h; j += 2) {
        float2 a = make_float2(v[blk + j], v[blk + j + 1]);
        float2 b = make_float2(v[blk + j + h], v[blk + j + h + 1]);
        float2 s = add2(a, b);
        float2 d = sub2(a, b);
        v[blk + j] = s.x;
        v[blk + j + 1] = s.y;
        v[blk + j + h] = d.x;
        v[blk + j + h + 1] = d.y;
      }
    }
  }
}

// One cross-lane butterfly stage.  Before: slot j of this lane is element
// (lane-group base) + j for the stage's lower partner, or the matching upper
// element.  The two partners swap the slot halves they will not finish; after
// the stage slot m (< EPL/2) holds the sum and slot EPL/2 + m the difference of
// pair m of the half this lane kept.
template <int EPL>
ASTERQ_DEVICE void fwht_cross_stage(float (&v)[EPL], int partner_mask, bool upper) {
  constexpr int HALF = EPL / 2;
#pragma unroll
  for (int m = 0; m < HALF; ++m) {
    float mine = upper ? v[HALF + m] : v[m];
    float send = upper ? v[m] : v[HALF + m];
    float recv = __shfl_xor_sync(0xffffffffu, send, partner_mask);
    // lower partner holds a (index bit = 0), upper holds b.
    float a = upper ? recv : mine;
    float b = upper ? mine : recv;
    v[m] = a + b;
    v[HALF + m] = a - b;
  }
}

// element i of the lane's slice lives at element index q*EPL + i
template <int EPL, int DT>
ASTERQ_DEVICE void load_slice(float (&v)[EPL], const void* row, int elem0, int dim_in, bool vec_ok) {
  if (DT == ASTERQ_DTYPE_BF16 || DT == ASTERQ_DTYPE_F16) {
    const uint16_t* p = reinterpret_cast<const uint16_t*>(row) + elem0;
    if (vec_ok) {
#pragma unroll
      for (int i = 0; i < EPL; i += 8) {
        uint4 w = ldg_nc_v4(p + i);
        uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (DT == ASTERQ_DTYPE_BF16) {
            v[i + 2 * k] = bf16lo_to_f32(ws[k]);
            v[i + 2 * k + 1] = bf16hi_to_f32(ws[k]);
          } else {
            float2 f = unpack_half2(ws[k]);
            v[i + 2 * k] = f.x;
            v[i + 2 * k + 1] = f.y;
          }
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        int e = elem0 + i;
        uint16_t b = (e < dim_in) ? p[i] : (uint16_t)0;
        if (DT == ASTERQ_DTYPE_BF16) {
          v[i] = __uint_as_float(((uint32_t)b) << 16);
        } else {
          v[i] = __half2float(__ushort_as_half(b));
        }
      }
    }
  } else {
    const float* p = reinterpret_cast<const float*>(row) + elem0;
    if (vec_ok) {
#pragma unroll
      for (int i = 0; i < EPL; i += 4) {
        uint4 w = ldg_nc_v4(p + i);
        v[i] = __uint_as_float(w.x);
        v[i + 1] = __uint_as_float(w.y);
        v[i + 2] = __uint_as_float(w.z);
        v[i + 3] = __uint_as_float(w.w);
      }
    } else {
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        int e = elem0 + i;
        v[i] = (e < dim_in) ? p[i] : 0.0f;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// K1: encode
// ---------------------------------------------------------------------------
// D: register width (power of two).  For hadamard_int4 it is the padded dim; for
// int4/int8 it is the smallest power of two >= the group-padded dim.
template <int D, int G, bool ROT, int QMAX, int DT>
__global__ void __launch_bounds__(256) encode_kernel(const void* __restrict__ x, int64_t n_tokens, int dim_in,
                                                     int64_t x_stride, int dim_out, uint8_t* __restrict__ codes,
                                                     __half* __restrict__ scales) {
  constexpr int EPL = D < 128 ? D : 128;
  constexpr int LPT = D / EPL;
  constexpr int TPW = 32 / LPT;
  constexpr int HALF = (LPT > 1) ? EPL / 2 : EPL;  // lane-local contiguous run after the cross stages
  static_assert(G <= HALF || (LPT == 1 && G <= EPL), "group must be lane-local");
  static_assert(HALF % G == 0, "group must divide the lane-local run");
  constexpr bool INT4 = (QMAX == 7);
  constexpr int ELEM_SIZE = (DT == ASTERQ_DTYPE_F32) ? 4 : 2;

  const int lane = threadIdx.x & 31;
  const int q = lane % LPT;
  const int t_in_warp = lane / LPT;
  const int64_t warp_id = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t n_warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int groups_out = dim_out / G;
  const int code_row_bytes = INT4 ? dim_out / 2 : dim_out;

  const float c = ROT ? kSqrtTable[__ffs(D) - 1] : 1.0f;  // float32(sqrt(D))
  const float rc = __frcp_rn(c);
  const bool vec_ok = (dim_in == D) && ((x_stride * ELEM_SIZE) % 16 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);

  for (int64_t base = warp_id * TPW; base < n_tokens; base += n_warps * TPW) {
    const int64_t tok = base + t_in_warp;
    const bool valid = tok < n_tokens;
    float v[EPL];
    if (valid) {
      const char* row = reinterpret_cast<const char*>(x) + tok * x_stride * ELEM_SIZE;
      load_slice<EPL, DT>(v, row, q * EPL, dim_in, vec_ok);
    } else {
#pragma unroll
      for (int i = 0; i < EPL; ++i) v[i] = 0.0f;
    }

    int elem_of_slot0_lo;  // element index of slot 0
    int elem_stride_hi;    // element offset of slot HALF relative to slot 0
    if (ROT) {
      fwht_local<EPL>(v);
#pragma unroll
      for (int s = 0; (1 << s) < LPT; ++s) {
        fwht_cross_stage<EPL>(v, 1 << s, ((q >> s) & 1) != 0);
      }
    }
    if (ROT && LPT > 1) {
      // slot t*HALF + m  <->  element m + HALF*(q + LPT*t)
      elem_of_slot0_lo = HALF * q;
      elem_stride_hi = HALF * LPT;
    } else {
      elem_of_slot0_lo = EPL * q;
      elem_stride_hi = HALF;
    }

    constexpr int NG = EPL / G;  // groups per lane
#pragma unroll
    for (int gi = 0; gi < NG; ++gi) {
      const int slot0 = gi * G;
      const int elem0 = elem_of_slot0_lo + (slot0 / HALF) * elem_stride_hi + (slot0 % HALF);
      const int gidx = elem0 / G;
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < G; ++i) amax = fmaxf(amax, fabsf(v[slot0 + i]));
      // amax of RN(y / c) equals RN(amax(y) / c): division by c > 0 and rounding
      // are both monotone, so one correctly rounded division per group suffices.
      const float amax_v = ROT ? __fdiv_rn(amax, c) : amax;
      const float scale = __fdiv_rn(fmaxf(amax_v, 1e-8f), (float)QMAX);
      const float rs = __frcp_rn(scale);
      // code = rint(RN(RN(y / c) / scale)): both quotients correctly rounded
      // (div_markstein), then adding 1.5*2^23 (+8 for the int4 offset) rounds to an
      // integer with ties to even exactly like rint() and leaves it in the low
      // mantissa bits.  |RN(v / scale)| <= 7 (resp. 127), so no clamp is needed.
      const float magic = INT4 ? 12582920.0f : 12582912.0f;
      constexpr int NW = INT4 ? G / 8 : G / 4;
      uint32_t words[NW];
#pragma unroll
      for (int w = 0; w < NW; ++w) words[w] = 0u;
#pragma unroll
      for (int i = 0; i < G; ++i) {
        const float y = v[slot0 + i];
        // Outside Markstein's exact range |y| < 2^-100, so |RN(y/c) / scale| <
        // 2^-70 (scale >= 1e-8/7) and the code is 0 either way: no fallback needed.
        const float vq = ROT ? div_markstein(y, c, rc) : y;
        const uint32_t ub = __float_as_uint(div_markstein(vq, scale, rs) + magic);
        if (INT4) {
          words[i >> 3] |= (ub & 0xFu) << (4 * (i & 7));
        } else {
          words[i >> 2] |= (ub & 0xFFu) << (8 * (i & 3));
        }
      }
      if (valid && gidx < groups_out) {
        uint8_t* crow = codes + tok * (int64_t)code_row_bytes;
        uint8_t* dst = crow + (INT4 ? elem0 / 2 : elem0);
        // byte k = u[2k] | u[2k+1] << 4 (kv.py:47-48); int8 codes as two's complement bytes
        if (NW >= 4) {
#pragma unroll
          for (int w = 0; w < NW; w += 4)
            *reinterpret_cast<uint4*>(dst + 4 * w) = make_uint4(words[w], words[w + 1], words[w + 2], words[w + 3]);
        } else if (NW == 2) {
          *reinterpret_cast<uint2*>(dst) = make_uint2(words[0], words[1]);
        } else {
          *reinterpret_cast<uint32_t*>(dst) = words[0];
        }
        scales[tok * (int64_t)groups_out + gidx] = __float2half_rn(scale);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// K1b: encode in the latent cache's own layout -- 512 bf16 values per token,
// hadamard_int4, groups of 16/32/64, 16-byte aligned rows.
//
// Each warp streams tiles of 4 tokens through a private 3-stage shared-memory
// ring filled by cp.async.bulk (one 1 KB copy per token row, completion on an
// mbarrier), so two further tiles are in flight while one is transformed; 16
// warps per SM.  Eight lanes own a token.  Lane l starts with elements
// 64 l + [0, 64) as eight blocks of 8; block k sits at register position
// p = k ^ l.  With that placement every butterfly partner is at a register
// position that does not depend on the lane:
//   bits 0-2  inside a block;
//   bits 3-5  positions p and p ^ 1 (p ^ 2, p ^ 4); which of the two holds the
//             lower element depends on the lane, absorbed by a per-position
//             storage sign (pos_stage);
//   exchange  position p moves to lane l ^ p (seven xor shuffles, no selects);
//   bits 6-8  as bits 3-5, on the exchanged blocks.
// Afterwards lane l holds elements 64 b + 8 l + [0, 8) at position b ^ l.  A
// group's absmax is reduced by recursive halving (7 shuffles for groups of 64),
// which leaves each lane owning whole groups; the owner computes the scale once
// and the other lanes fetch it.  The XOR placement also spreads each 16-byte
// shared-memory read of a warp evenly over the banks (4 wavefronts per 512 bytes).
//
// Divisions.  RN(y / c) for c = float32(sqrt(512)) is RN(y*ch + RN(y*cl)) with
// ch = RN(1/c), cl = RN(1/c - ch) (Brisebarre and Muller, "Correctly rounded
// multiplication by arbitrary precision constants", IEEE Trans. Computers 57(2),
// 2008); tests/div_check.c checks it over every significand.  Division by the
// group scale (and of the absmax by 7) keeps Markstein's correction step.  Both
// are exact for 2^-98 <= |y| <= 2^120; below that range the code is 0 either way,
// and a tile holding a group whose absmax is above 2^119 (or not finite) takes
// IEEE divisions throughout.
// ---------------------------------------------------------------------------
namespace lat512 {
constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 3;
constexpr int kTok = 4;                        // tokens per warp tile
constexpr int kRowBytes = 1024;                // one bf16 token row
constexpr int kStageBytes = kTok * kRowBytes;  // 4 KB: rows back to back
constexpr int kWarpBytes = kStages * kStageBytes;
constexpr int kBarOff = kWarps * kWarpBytes;   // 196,608
constexpr int kSmem = kBarOff + kWarps * kStages * 8 + 16;
constexpr float kC = 0x1.6a09e6p+4f;           // float32(sqrt(512))
constexpr float kCh = 0x1.6a09e6p-5f;          // RN(1 / kC)
constexpr float kCl = 0x1.9fcef4p-30f;         // RN(1 / kC - kCh)
constexpr float kR7 = 0x1.24924ap-3f;          // RN(1 / 7)
}  // namespace lat512

__device__ int g_codec_timeouts;  // encode waits that gave up (read by asterq_codec_status)

ASTERQ_DEVICE uint4 lds128(uint32_t addr) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr) : "memory");
  return r;
}

// (a, b) -> (a + b, a - b) for two neighbouring pairs at once
ASTERQ_DEVICE void bfly_pair(float& a0, float& a1, float& b0, float& b1) {
  const float2 A = make_float2(a0, a1), B = make_float2(b0, b1);
  const float2 s = add2(A, B), d = sub2(A, B);
  a0 = s.x; a1 = s.y; b0 = d.x; b1 = d.y;
}

// Butterflies on element-index bit log2(H) (H = 2, 4), inside every block of 8.
template <int H>
ASTERQ_DEVICE void block_stage(float (&x)[64]) {
#pragma unroll
  for (int base = 0; base < 64; base += 2 * H) {
#pragma unroll
    for (int j = 0; j < H; j += 2) bfly_pair(x[base + j], x[base + j + 1], x[base + j + H], x[base + j + H + 1]);
  }
}

// Butterflies between register positions p and p ^ M (blocks of 8), the same
// add and subtract in every lane.  Which of the two positions holds the lower
// element depends on the lane; that is absorbed by storing position p negated
// when parity(p & l) is odd.  With A = s a and B = s b (p holds the lower a),
// A + B = s (a + b) and A - B = s (a - b); with A = -s b and B = s a (p holds the
// upper b), A + B = s (a - b) and A - B = -s (a + b): each output is the
// reference's single rounding, up to a sign.  The upper case flips every sign of
// the lane at once, which keeps the parity pattern; the exchange between phases
// preserves it too (received position q carries parity(q & ~l) + popcount(l ^ q),
// which equals parity(q & l) + popcount(l) mod 2), so after all six stages
// position q holds (-1)^parity(q & l) times the true outputs.
template <int M>
ASTERQ_DEVICE void pos_stage(float (&x)[64]) {
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    if (p & M) continue;
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      bfly_pair(x[p * 8 + i], x[p * 8 + i + 1], x[(p ^ M) * 8 + i], x[(p ^ M) * 8 + i + 1]);
    }
  }
}

constexpr float kMagic = 12582920.0f;  // 1.5 * 2^23 + 8: rounds to an integer, ties to even, plus the int4 offset
constexpr float kTieGuard = 0.5f - 0x1p-16f;

// One byte from the low nibbles of t0 (even element) and t1 (odd element):
// t0 + 16 * t1, whose low byte is u0 | u1 << 4 (kv.py:47-48) as both low bytes
// hold q + 8 in [1, 15].
ASTERQ_DEVICE uint32_t pack_pair(float t0, float t1) {
  uint32_t r;
  asm("mad.lo.u32 %0, %1, 16, %2;" : "=r"(r) : "r"(__float_as_uint(t1)), "r"(__float_as_uint(t0)));
  return r;
}
ASTERQ_DEVICE uint32_t pack_word(const uint32_t (&by)[4]) {
  return prmt(prmt(by[0], by[1], 0x0040u), prmt(by[2], by[3], 0x0040u), 0x5410u);
}

// Codes of one block of 8 elements exactly as the reference rounds them,
// rint(RN(RN(y / c) / sc)), packed into one word.  rs = RN(1 / sc).
template <bool IEEE>
ASTERQ_DEVICE uint32_t quantize8(const float* y, float sc, float rs) {
  uint32_t by[4];
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    float t0, t1;
    if (IEEE) {
      t0 = __fadd_rn(__fdiv_rn(__fdiv_rn(y[i], lat512::kC), sc), kMagic);
      t1 = __fadd_rn(__fdiv_rn(__fdiv_rn(y[i + 1], lat512::kC), sc), kMagic);
    } else {
      const float2 Y = make_float2(y[i], y[i + 1]);
      const float2 vq = fma2(Y, make_float2(lat512::kCh, lat512::kCh), mul2(Y, make_float2(lat512::kCl, lat512::kCl)));
      const float2 r2 = make_float2(rs, rs);
      const float2 q0 = mul2(vq, r2);
      const float2 e = fma2(q0, make_float2(-sc, -sc), vq);
      const float2 q1 = fma2(e, r2, q0);
      const float2 t = add2(q1, make_float2(kMagic, kMagic));
      t0 = t.x;
      t1 = t.y;
    }
    by[i / 2] = pack_pair(t0, t1);
  }
  return pack_word(by);
}

// Candidate codes rint(y * k) for k = RN(1 / RN(c * sc)), packed into one word,
// with max |y*k - rint(y*k)| folded into dmax.  The exact product y*k is within
// a relative 2^-22 of the reference's RN(RN(y / c) / sc) (|value| <= 7), so where
// it lies farther than 2^-16 from every half-integer (dmax < kTieGuard) both
// round to the same integer; otherwise the caller recomputes with quantize8.
ASTERQ_DEVICE uint32_t quantize8_fast(const float* y, float k, float& dmax) {
  const float2 k2 = make_float2(k, k), m2 = make_float2(kMagic, kMagic);
  uint32_t by[4];
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    const float2 Y = make_float2(y[i], y[i + 1]);
    const float2 t = fma2(Y, k2, m2);   // kMagic + rint(y*k), one rounding of the exact y*k + kMagic
    const float2 nq = sub2(m2, t);      // -rint(y*k), exact
    const float2 d = fma2(Y, k2, nq);   // y*k - rint(y*k)
    dmax = fmaxf(dmax, fmaxf(fabsf(d.x), fabsf(d.y)));
    by[i / 2] = pack_pair(t.x, t.y);
  }
  return pack_word(by);
}

// Scale of one group from the absmax of its (unnormalized) transform outputs:
// RN(max(RN(amax / c), 1e-8) / 7) (kv.py:104-106).
template <bool IEEE>
ASTERQ_DEVICE float group_scale(float amax) {
  if (IEEE) return __fdiv_rn(fmaxf(__fdiv_rn(amax, lat512::kC), 1e-8f), 7.0f);
  const float av = fmaf(amax, lat512::kCh, __fmul_rn(amax, lat512::kCl));
  const float m = fmaxf(av, 1e-8f);
  const float q0 = __fmul_rn(m, lat512::kR7);
  return fmaf(fmaf(-q0, 7.0f, m), lat512::kR7, q0);
}

// f negated where the position's storage sign is negative.  A negated divisor (or
// factor) undoes the stored negation exactly: RN(-a / -s) = RN(a / s).
ASTERQ_DEVICE float signed_by(float f, uint32_t negmask) { return __uint_as_float(__float_as_uint(f) ^ (negmask << 16)); }

ASTERQ_DEVICE void mbar_drain(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try(bar, parity) && clock64() - t0 < 4000000000LL) {
  }
}

template <int G>
__global__ void __launch_bounds__(lat512::kThreads, 1)
    encode_lat512_kernel(const uint16_t* __restrict__ x, int64_t n_tokens, int64_t x_stride,
                         uint8_t* __restrict__ codes, __half* __restrict__ scales) {
  using namespace lat512;
  constexpr int LPG = G / 8;       // lanes sharing a group
  constexpr int OWN = 8 / LPG;     // groups owned per lane after the reduction
  constexpr int GPT = 512 / G;     // groups per token
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = lane >> 3, l = lane & 7;
  const uint32_t ring = smem_u32(smem) + warp * kWarpBytes;
  const uint32_t bar0 = smem_u32(smem + kBarOff) + warp * kStages * 8;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kBarOff + kWarps * kStages * 8);
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) mbar_init(bar0 + 8 * s, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (threadIdx.x == 0) *abort_flag = 0;
  __syncthreads();

  const int64_t n_tiles = (n_tokens + kTok - 1) / kTok;
  const int64_t first = (int64_t)blockIdx.x * kWarps + warp;
  const int64_t step = (int64_t)gridDim.x * kWarps;
  auto issue = [&](int64_t tile, int s) {
    const int64_t tok0 = tile * kTok;
    const int nv = (int)((n_tokens - tok0) < kTok ? (n_tokens - tok0) : kTok);
    if (lane == 0) mbar_expect_tx(bar0 + 8 * s, (uint32_t)(nv * kRowBytes));
    __syncwarp();
    if (x_stride == 512) {  // contiguous rows: one copy for the tile
      if (lane == 0) bulk_1d(ring + s * kStageBytes, x + tok0 * 512, (uint32_t)(nv * kRowBytes), bar0 + 8 * s);
    } else if (lane < nv) {
      bulk_1d(ring + s * kStageBytes + lane * kRowBytes, x + (tok0 + lane) * x_stride, kRowBytes, bar0 + 8 * s);
    }
  };
#pragma unroll
  for (int s = 0; s < kStages; ++s)
    if (first + s * step < n_tiles) issue(first + s * step, s);

  // Long launches: start the four warps of each scheduler a microsecond apart so
  // their FMA-heavy and ALU-heavy phases overlap instead of coinciding.
  if (n_tiles >= 8 * step) __nanosleep(1000u * (unsigned)(warp >> 2));
  uint32_t negm[8];  // 0x80008000 where parity(p & l) is odd: position p is stored negated
#pragma unroll
  for (int p = 0; p < 8; ++p) negm[p] = (__popc(p & l) & 1) ? 0x80008000u : 0u;
  int64_t it = 0;
  for (;; ++it) {
    const int64_t tile = first + it * step;
    if (tile >= n_tiles) break;
    const int s = (int)(it % kStages);
    const uint32_t parity = (uint32_t)((it / kStages) & 1);
    if (!mbar_wait(bar0 + 8 * s, parity, abort_flag)) break;
    const int64_t tok = tile * kTok + t;
    const bool valid = tok < n_tokens;

    // load with butterfly stage h = 1 (element pairs 2m, 2m + 1 are one bf16x2 word)
    float v[64];
    {
      const uint32_t row = ring + s * kStageBytes + t * kRowBytes + 128 * l;
      uint4 w[8];
#pragma unroll
      for (int p = 0; p < 8; ++p) w[p] = lds128(row + 16 * (p ^ l));
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        const uint32_t ws[4] = {w[p].x, w[p].y, w[p].z, w[p].w};
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          // lo + hi and lo - hi (negated for the position's storage sign) with lo read
          // as bf16 straight from the word's low half: bf16 -> f32 is exact, so each
          // is the reference's single f32 rounding
          const uint32_t w2 = ws[m] ^ negm[p];
          float s0, s1;
          asm("{\n .reg .b16 lo, hi;\n mov.b32 {lo, hi}, %2;\n add.rn.f32.bf16 %0, lo, %3;\n sub.rn.f32.bf16 %1, lo, %3;\n}"
              : "=f"(s0), "=f"(s1)
              : "r"(w2), "f"(bf16hi_to_f32(w2)));
          v[p * 8 + 2 * m] = s0;
          v[p * 8 + 2 * m + 1] = s1;
        }
      }
    }
    // every lane's copy of the stage is in registers: refill it with the tile kStages ahead
    __syncwarp();
    fence_async_shared();
    if (tile + kStages * step < n_tiles) issue(tile + kStages * step, s);

    block_stage<2>(v);
    block_stage<4>(v);
    pos_stage<1>(v);
    pos_stage<2>(v);
    pos_stage<4>(v);
#pragma unroll
    for (int p = 1; p < 8; ++p) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[p * 8 + i] = __shfl_xor_sync(0xffffffffu, v[p * 8 + i], p);
    }
    pos_stage<1>(v);
    pos_stage<2>(v);
    pos_stage<4>(v);

    // absmax of each block, then recursive halving over the LPG lanes of a group:
    // lane l ^ m keeps the same block at position q ^ m, so after the round for m
    // the positions with bit m clear hold the maximum over both lanes
    float am[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float a = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) a = fmaxf(a, fabsf(v[q * 8 + i]));
      am[q] = a;
    }
#pragma unroll
    for (int m = LPG / 2; m >= 1; m /= 2) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if ((q & (LPG - 1)) >= m) continue;  // still active and bit m clear
        am[q] = fmaxf(am[q], __shfl_xor_sync(0xffffffffu, am[q ^ m], m));
      }
    }
    // this lane owns the groups at positions q with q & (LPG - 1) == 0
    bool big = false;
#pragma unroll
    for (int o = 0; o < OWN; ++o) big |= !(am[o * LPG] <= 0x1p119f);
    big = big && valid;
    const bool ieee = __any_sync(0xffffffffu, big);
    float osc[OWN];
#pragma unroll
    for (int o = 0; o < OWN; ++o) osc[o] = ieee ? group_scale<true>(am[o * LPG]) : group_scale<false>(am[o * LPG]);
    // position q's group is owned by lane l ^ (q & (LPG - 1)) at its position q & ~(LPG - 1)
    auto fetch = [&](const float (&own)[OWN], int q) {
      const int m = q & (LPG - 1);
      return m ? __shfl_xor_sync(0xffffffffu, own[q / LPG], m) : own[q / LPG];
    };
    uint32_t cw[8];
    if (!ieee) {
      float ok[OWN];
#pragma unroll
      for (int o = 0; o < OWN; ++o) ok[o] = __frcp_rn(__fmul_rn(kC, osc[o]));
      float dmax = 0.0f;
#pragma unroll
      for (int q = 0; q < 8; ++q) cw[q] = quantize8_fast(v + q * 8, signed_by(fetch(ok, q), negm[q]), dmax);
      if (__any_sync(0xffffffffu, valid && !(dmax < kTieGuard))) {
        // a value within 2^-16 of a half-integer somewhere in the tile: redo the tile exactly
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float sc = signed_by(fetch(osc, q), negm[q]);
          cw[q] = quantize8<false>(v + q * 8, sc, __frcp_rn(sc));
        }
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) cw[q] = quantize8<true>(v + q * 8, signed_by(fetch(osc, q), negm[q]), 0.0f);
    }
    if (valid) {
      // block b = q ^ l holds elements 64 b + 8 l + [0, 8): code bytes 32 b + 4 l
      uint8_t* crow = codes + tok * 256 + 4 * l;
#pragma unroll
      for (int q = 0; q < 8; ++q) *reinterpret_cast<uint32_t*>(crow + 32 * (q ^ l)) = cw[q];
#pragma unroll
      for (int o = 0; o < OWN; ++o) {
        const int g = (64 * ((o * LPG) ^ l) + 8 * l) / G;
        scales[tok * GPT + g] = __float2half_rn(osc[o]);
      }
    }
  }
  if (*abort_flag) {
    // a copy never completed: record it and wait (bounded) for this warp's copies still in flight
    if (lane == 0) atomicAdd(&g_codec_timeouts, 1);
    for (int64_t k = it; k < it + kStages; ++k) {
      const int64_t tile = first + k * step;
      if (tile >= n_tiles) break;
      mbar_drain(bar0 + 8 * (int)(k % kStages), (uint32_t)((k / kStages) & 1));
    }
  }
}

// ---------------------------------------------------------------------------
// Dequantize (kv.py:121-134): restored = codes * float(scale), inverse FWHT,
// crop, cast.  Bit-exact for hadamard_int4 / int4 / int8.
// ---------------------------------------------------------------------------
template <int D, int G, bool ROT, int QMAX>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ codes, const __half* __restrict__ scales,
                                                     int64_t n_tokens, int dim_code, int dim_out, void* __restrict__ out,
                                                     int out_dtype, int64_t out_stride) {
  constexpr int EPL = D < 128 ? D : 128;
  constexpr int LPT = D / EPL;
  constexpr int TPW = 32 / LPT;
  constexpr int HALF = (LPT > 1) ? EPL / 2 : EPL;
  constexpr bool INT4 = (QMAX == 7);

  const int lane = threadIdx.x & 31;
  const int q = lane % LPT;
  const int t_in_warp = lane / LPT;
  const int64_t warp_id = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t n_warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int groups = dim_code / G;
  const int code_row_bytes = INT4 ? dim_code / 2 : dim_code;
  const float c = ROT ? kSqrtTable[__ffs(D) - 1] : 1.0f;
  const float rc = ROT ? __frcp_rn(c) : 1.0f;

  for (int64_t base = warp_id * TPW; base < n_tokens; base += n_warps * TPW) {
    const int64_t tok = base + t_in_warp;
    const bool valid = tok < n_tokens;
    float v[EPL];
    // slot i <-> element q*EPL + i (the natural order before the transform)
#pragma unroll
    for (int g0 = 0; g0 < EPL; g0 += G) {
      const int e0 = q * EPL + g0;
      const int gidx = e0 / G;
      if (valid && gidx < groups) {
        const float s = __half2float(scales[tok * (int64_t)groups + gidx]);
        const uint8_t* crow = codes + tok * (int64_t)code_row_bytes;
#pragma unroll
        for (int i = 0; i < G; ++i) {
          int code;
          if (INT4) {
            const uint8_t b = crow[(e0 + i) >> 1];
            code = (int)(((i & 1) ? (b >> 4) : b) & 0xF) - 8;
          } else {
            code = (int)(int8_t)crow[e0 + i];
          }
          v[g0 + i] = (float)code * s;
        }
      } else {
#pragma unroll
        for (int i = 0; i < G; ++i) v[g0 + i] = 0.0f;
      }
    }
    int elem_of_slot0_lo = EPL * q, elem_stride_hi = HALF;
    if (ROT) {
      fwht_local<EPL>(v);
#pragma unroll
      for (int s = 0; (1 << s) < LPT; ++s) fwht_cross_stage<EPL>(v, 1 << s, ((q >> s) & 1) != 0);
      if (LPT > 1) {
        elem_of_slot0_lo = HALF * q;
        elem_stride_hi = HALF * LPT;
      }
#pragma unroll
      for (int i = 0; i < EPL; ++i) v[i] = div_by_const(v[i], c, rc);
    }
    if (!valid) continue;
    char* orow = reinterpret_cast<char*>(out);
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = elem_of_slot0_lo + (i / HALF) * elem_stride_hi + (i % HALF);
      if (e >= dim_out) continue;
      const int64_t off = tok * out_stride + e;
      if (out_dtype == ASTERQ_DTYPE_F32) {
        reinterpret_cast<float*>(orow)[off] = v[i];
      } else if (out_dtype == ASTERQ_DTYPE_BF16) {
        reinterpret_cast<__nv_bfloat16*>(orow)[off] = __float2bfloat16_rn(v[i]);
      } else {
        reinterpret_cast<__half*>(orow)[off] = __float2half_rn(v[i]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Normalized FWHT of float32 rows (kv.py:13-32), bit-exact.
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) fwht_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t rows) {
  constexpr int EPL = D < 128 ? D : 128;
  constexpr int LPT = D / EPL;
  constexpr int TPW = 32 / LPT;
  constexpr int HALF = (LPT > 1) ? EPL / 2 : EPL;
  const int lane = threadIdx.x & 31;
  const int q = lane % LPT;
  const int t_in_warp = lane / LPT;
  const int64_t warp_id = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t n_warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const float c = kSqrtTable[__ffs(D) - 1];
  const float rc = __frcp_rn(c);
  for (int64_t base = warp_id * TPW; base < rows; base += n_warps * TPW) {
    const int64_t r = base + t_in_warp;
    const bool valid = r < rows;
    float v[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) v[i] = valid ? x[r * D + q * EPL + i] : 0.0f;
    fwht_local<EPL>(v);
#pragma unroll
    for (int s = 0; (1 << s) < LPT; ++s) fwht_cross_stage<EPL>(v, 1 << s, ((q >> s) & 1) != 0);
    if (!valid) continue;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = (LPT > 1) ? (i % HALF) + HALF * (q + LPT * (i / HALF)) : q * EPL + i;
      y[r * D + e] = div_by_const(v[i], c, rc);
    }
  }
}

// ---------------------------------------------------------------------------
// Host-side dispatch
// ---------------------------------------------------------------------------
namespace {

int grid_for(int64_t n_tokens, int tokens_per_block) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t blocks = (n_tokens + tokens_per_block - 1) / tokens_per_block;
  int64_t cap = (int64_t)sms * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

template <int D, int G, bool ROT, int QMAX>
int launch_encode_dt(const void* x, int x_dtype, int64_t n, int dim_in, int64_t stride, int dim_out, uint8_t* codes,
                     __half* scales, cudaStream_t st) {
  constexpr int EPL = D < 128 ? D : 128;
  constexpr int TPB = 8 * (32 / (D / EPL));
  const int grid = grid_for(n, TPB);
  switch (x_dtype) {
    case ASTERQ_DTYPE_BF16:
      encode_kernel<D, G, ROT, QMAX, ASTERQ_DTYPE_BF16><<<grid, 256, 0, st>>>(x, n, dim_in, stride, dim_out, codes, scales);
      break;
    case ASTERQ_DTYPE_F16:
      encode_kernel<D, G, ROT, QMAX, ASTERQ_DTYPE_F16><<<grid, 256, 0, st>>>(x, n, dim_in, stride, dim_out, codes, scales);
      break;
    case ASTERQ_DTYPE_F32:
      encode_kernel<D, G, ROT, QMAX, ASTERQ_DTYPE_F32><<<grid, 256, 0, st>>>(x, n, dim_in, stride, dim_out, codes, scales);
      break;
    default:
      return set_error(ASTERQ_ERR_UNSUPPORTED, "encode: unsupported source dtype %d", x_dtype);
  }
  return check_launch("encode");
}

template <int D, bool ROT, int QMAX>
int launch_encode_g(int G, const void* x, int x_dtype, int64_t n, int dim_in, int64_t stride, int dim_out,
                    uint8_t* codes, __half* scales, cudaStream_t st) {
  switch (G) {
    case 16:
      if constexpr (D >= 16)
        return launch_encode_dt<D, 16, ROT, QMAX>(x, x_dtype, n, dim_in, stride, dim_out, codes, scales, st);
      break;
    case 32:
      if constexpr (D >= 32 && (D <= 128 || D >= 64))
        return launch_encode_dt<D, 32, ROT, QMAX>(x, x_dtype, n, dim_in, stride, dim_out, codes, scales, st);
      break;
    case 64:
      if constexpr (D >= 64)
        return launch_encode_dt<D, 64, ROT, QMAX>(x, x_dtype, n, dim_in, stride, dim_out, codes, scales, st);
      break;
    default:
      break;
  }
  return set_error(ASTERQ_ERR_UNSUPPORTED, "encode: group_size %d unsupported for register width %d", G, D);
}

template <bool ROT, int QMAX>
int launch_encode_d(int D, int G, const void* x, int x_dtype, int64_t n, int dim_in, int64_t stride, int dim_out,
                    uint8_t* codes, __half* scales, cudaStream_t st) {
  switch (D) {
    case 16:
      return launch_encode_g<16, ROT, QMAX>(G, x, x_dtype, n, dim_in, stride, dim_out, codes, scales, st);
    case 32:
      return launch_encode_g<32, ROT, QMAX>(G, x, x_dtype, n, dim_in, stride, dim_out, codes, scales, st);
    case 64:
      return launch_encode_g<64, ROT, QMAX>(G, x, x_dtype, n, dim_in, stride, dim_out, codes, scales, st);
    case 128:
      return launch_encode_g<128, ROT, QMAX>(G, x, x_dtype, n, dim_in, stride, dim_out, codes, scales, st);
    case 256:
      return launch_encode_g<256, ROT, QMAX>(G, x, x_dtype, n, dim_in, stride, dim_out, codes, scales, st);
    case 512:
      return launch_encode_g<512, ROT, QMAX>(G, x, x_dtype, n, dim_in, stride, dim_out, codes, scales, st);
    default:
      return set_error(ASTERQ_ERR_UNSUPPORTED, "encode: padded width %d unsupported (16..512)", D);
  }
}

template <int G>
int launch_encode_lat512(const void* x, int64_t n, int64_t stride, uint8_t* codes, __half* scales, cudaStream_t st) {
  static int attr_set[64];  // per device: the kernel's dynamic shared memory limit is raised once
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  if (dev >= 64 || !attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(encode_lat512_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               lat512::kSmem);
    if (e != cudaSuccess) return set_error(ASTERQ_ERR_CUDA, "encode: %s", cudaGetErrorString(e));
    if (dev < 64) attr_set[dev] = 1;
  }
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t tiles = (n + lat512::kTok - 1) / lat512::kTok;
  int64_t blocks = (tiles + lat512::kWarps - 1) / lat512::kWarps;
  if (blocks > sms) blocks = sms;
  encode_lat512_kernel<G><<<(int)blocks, lat512::kThreads, lat512::kSmem, st>>>(
      reinterpret_cast<const uint16_t*>(x), n, stride, codes, scales);
  return check_launch("encode");
}

template <int D, int G, bool ROT, int QMAX>
int launch_decode_one(const uint8_t* codes, const __half* scales, int64_t n, int dim_code, int dim_out, void* out,
                      int out_dtype, int64_t out_stride, cudaStream_t st) {
  constexpr int EPL = D < 128 ? D : 128;
  constexpr int TPB = 8 * (32 / (D / EPL));
  dequant_kernel<D, G, ROT, QMAX><<<grid_for(n, TPB), 256, 0, st>>>(codes, scales, n, dim_code, dim_out, out, out_dtype,
                                                                 out_stride);
  return check_launch("decode");
}

template <int D, bool ROT, int QMAX>
int launch_decode_g(int G, const uint8_t* codes, const __half* scales, int64_t n, int dim_code, int dim_out, void* out,
                    int out_dtype, int64_t out_stride, cudaStream_t st) {
  switch (G) {
    case 16:
      if constexpr (D >= 16)
        return launch_decode_one<D, 16, ROT, QMAX>(codes, scales, n, dim_code, dim_out, out, out_dtype, out_stride, st);
      break;
    case 32:
      if constexpr (D >= 32)
        return launch_decode_one<D, 32, ROT, QMAX>(codes, scales, n, dim_code, dim_out, out, out_dtype, out_stride, st);
      break;
    case 64:
      if constexpr (D >= 64)
        return launch_decode_one<D, 64, ROT, QMAX>(codes, scales, n, dim_code, dim_out, out, out_dtype, out_stride, st);
      break;
    default:
      break;
  }
  return set_error(ASTERQ_ERR_UNSUPPORTED, "dequantize: group_size %d unsupported for register width %d", G, D);
}

template <bool ROT, int QMAX>
int launch_decode_d(int D, int G, const uint8_t* codes, const __half* scales, int64_t n, int dim_code, int dim_out,
                    void* out, int out_dtype, int64_t out_stride, cudaStream_t st) {
  switch (D) {
    case 16:
      return launch_decode_g<16, ROT, QMAX>(G, codes, scales, n, dim_code, dim_out, out, out_dtype, out_stride, st);
    case 32:
      return launch_decode_g<32, ROT, QMAX>(G, codes, scales, n, dim_code, dim_out, out, out_dtype, out_stride, st);
    case 64:
      return launch_decode_g<64, ROT, QMAX>(G, codes, scales, n, dim_code, dim_out, out, out_dtype, out_stride, st);
    case 128:
      return launch_decode_g<128, ROT, QMAX>(G, codes, scales, n, dim_code, dim_out, out, out_dtype, out_stride, st);
    case 256:
      return launch_decode_g<256, ROT, QMAX>(G, codes, scales, n, dim_code, dim_out, out, out_dtype, out_stride, st);
    case 512:
      return launch_decode_g<512, ROT, QMAX>(G, codes, scales, n, dim_code, dim_out, out, out_dtype, out_stride, st);
    default:
      return set_error(ASTERQ_ERR_UNSUPPORTED, "dequantize: width %d unsupported (16..512)", D);
  }
}

int pow2_at_least(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

// float8 (kv.py:85-89): x.to(torch.float8_e4m3fn), one byte a value, no scales.  One block
// per row at a time (rows grid-strided), threads over the row's values.
__global__ void __launch_bounds__(256) f8_encode_kernel(const void* __restrict__ x, int x_dtype, int64_t n_tokens,
                                                        int dim, int64_t stride, uint8_t* __restrict__ codes) {
  for (int64_t t = blockIdx.x; t < n_tokens; t += gridDim.x)
    for (int d = threadIdx.x; d < dim; d += blockDim.x) {
      const int64_t i = t * stride + d;
      float v;
      if (x_dtype == ASTERQ_DTYPE_F32) v = reinterpret_cast<const float*>(x)[i];
      else if (x_dtype == ASTERQ_DTYPE_BF16) v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]);
      else v = __half2float(reinterpret_cast<const __half*>(x)[i]);
      codes[t * dim + d] = (uint8_t)f32_to_e4m3(v);
    }
}

// the e4m3 values widened to out_dtype (exact in fp32, bf16 and fp16)
__global__ void __launch_bounds__(256) f8_decode_kernel(const uint8_t* __restrict__ codes, int64_t n_tokens, int dim,
                                                        void* __restrict__ out, int out_dtype, int64_t out_stride) {
  for (int64_t t = blockIdx.x; t < n_tokens; t += gridDim.x)
    for (int d = threadIdx.x; d < dim; d += blockDim.x) {
      const uint32_t c = codes[t * dim + d];
      const float v = __half2float(__ushort_as_half((unsigned short)(e4m3x2_to_f16x2(c | (c << 8)) & 0xFFFFu)));
      const int64_t i = t * out_stride + d;
      if (out_dtype == ASTERQ_DTYPE_F32) reinterpret_cast<float*>(out)[i] = v;
      else if (out_dtype == ASTERQ_DTYPE_BF16) reinterpret_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
      else reinterpret_cast<__half*>(out)[i] = __float2half_rn(v);
    }
}

int f8_grid(int64_t n_tokens) { return (int)(n_tokens < 148 * 16 ? n_tokens : 148 * 16); }

}  // namespace

}  // namespace asterq

using namespace asterq;

extern "C" int asterq_quantize(const void* x, int x_dtype, int64_t n_tokens, int dim, int64_t x_row_stride,
                               int scheme, int group_size, void* codes, void* scales, void* stream) {
  clear_error();
  if (n_tokens < 0 || dim <= 0 || group_size <= 0)
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "quantize: bad sizes (n_tokens=%lld dim=%d group=%d)",
                     (long long)n_tokens, dim, group_size);
  if (x_row_stride < dim) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "quantize: row stride %lld < dim %d",
                                           (long long)x_row_stride, dim);
  if (n_tokens == 0) return ASTERQ_OK;
  if (!x || !codes || (!scales && scheme != ASTERQ_SCHEME_FLOAT8))
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "quantize: null pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (scheme == ASTERQ_SCHEME_FLOAT8) {
    if (x_dtype != ASTERQ_DTYPE_F32 && x_dtype != ASTERQ_DTYPE_BF16 && x_dtype != ASTERQ_DTYPE_F16)
      return set_error(ASTERQ_ERR_UNSUPPORTED, "quantize: float8 from dtype %d unsupported", x_dtype);
    f8_encode_kernel<<<f8_grid(n_tokens), 256, 0, st>>>(x, x_dtype, n_tokens, dim, x_row_stride,
                                                        reinterpret_cast<uint8_t*>(codes));
    return check_launch("encode (float8)");
  }
  if (scheme == ASTERQ_SCHEME_HADAMARD_INT4) {
    const int padded = pow2_at_least(dim);
    if (padded % group_size) return set_error(ASTERQ_ERR_UNSUPPORTED, "quantize: group %d does not divide %d", group_size, padded);
    if ((reinterpret_cast<uintptr_t>(codes) & 15) || (reinterpret_cast<uintptr_t>(scales) & 1))
      return set_error(ASTERQ_ERR_MISALIGNED, "quantize: codes must be 16-byte aligned");
    // the cache's own rows (512 bf16 values, 16-byte aligned) take the TMA-fed kernel
    if (dim == 512 && x_dtype == ASTERQ_DTYPE_BF16 && !(reinterpret_cast<uintptr_t>(x) & 15) && x_row_stride % 8 == 0 &&
        !(reinterpret_cast<uintptr_t>(scales) & 15)) {
      uint8_t* c8 = reinterpret_cast<uint8_t*>(codes);
      __half* sh = reinterpret_cast<__half*>(scales);
      if (group_size == 64) return launch_encode_lat512<64>(x, n_tokens, x_row_stride, c8, sh, st);
      if (group_size == 32) return launch_encode_lat512<32>(x, n_tokens, x_row_stride, c8, sh, st);
      if (group_size == 16) return launch_encode_lat512<16>(x, n_tokens, x_row_stride, c8, sh, st);
    }
    return launch_encode_d<true, 7>(padded, group_size, x, x_dtype, n_tokens, dim, x_row_stride, padded,
                                    reinterpret_cast<uint8_t*>(codes), reinterpret_cast<__half*>(scales), st);
  }
  if (scheme == ASTERQ_SCHEME_INT4 || scheme == ASTERQ_SCHEME_INT8) {
    const int dim_out = ((dim + group_size - 1) / group_size) * group_size;
    const int width = pow2_at_least(dim_out);
    // each group's codes are written with stores of min(16, group bytes) bytes
    const int row_bytes = (scheme == ASTERQ_SCHEME_INT4) ? dim_out / 2 : dim_out;
    const int group_bytes = (scheme == ASTERQ_SCHEME_INT4) ? group_size / 2 : group_size;
    const int chunk = group_bytes < 16 ? group_bytes : 16;
    if ((reinterpret_cast<uintptr_t>(codes) % chunk) || (row_bytes % chunk))
      return set_error(ASTERQ_ERR_MISALIGNED, "quantize: codes (row of %d bytes) must be %d-byte aligned", row_bytes, chunk);
    if (scheme == ASTERQ_SCHEME_INT4)
      return launch_encode_d<false, 7>(width, group_size, x, x_dtype, n_tokens, dim, x_row_stride, dim_out,
                                       reinterpret_cast<uint8_t*>(codes), reinterpret_cast<__half*>(scales), st);
    return launch_encode_d<false, 127>(width, group_size, x, x_dtype, n_tokens, dim, x_row_stride, dim_out,
                                       reinterpret_cast<uint8_t*>(codes), reinterpret_cast<__half*>(scales), st);
  }
  return set_error(ASTERQ_ERR_UNSUPPORTED, "quantize: unsupported scheme %d", scheme);
}

extern "C" int asterq_dequantize(const void* codes, const void* scales, int64_t n_tokens, int dim, int scheme,
                                 int group_size, void* out, int out_dtype, int64_t out_row_stride, void* stream) {
  clear_error();
  if (n_tokens < 0 || dim <= 0 || group_size <= 0 || out_row_stride < dim)
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "dequantize: bad sizes");
  if (n_tokens == 0) return ASTERQ_OK;
  if (!codes || (!scales && scheme != ASTERQ_SCHEME_FLOAT8) || !out)
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "dequantize: null pointer");
  if (out_dtype != ASTERQ_DTYPE_F32 && out_dtype != ASTERQ_DTYPE_BF16 && out_dtype != ASTERQ_DTYPE_F16)
    return set_error(ASTERQ_ERR_UNSUPPORTED, "dequantize: unsupported output dtype %d", out_dtype);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (scheme == ASTERQ_SCHEME_FLOAT8) {
    f8_decode_kernel<<<f8_grid(n_tokens), 256, 0, st>>>(reinterpret_cast<const uint8_t*>(codes), n_tokens, dim, out,
                                                        out_dtype, out_row_stride);
    return check_launch("decode (float8)");
  }
  if (scheme == ASTERQ_SCHEME_HADAMARD_INT4) {
    const int padded = pow2_at_least(dim);
    if (padded % group_size) return set_error(ASTERQ_ERR_UNSUPPORTED, "dequantize: group %d does not divide %d", group_size, padded);
    return launch_decode_d<true, 7>(padded, group_size, reinterpret_cast<const uint8_t*>(codes),
                                    reinterpret_cast<const __half*>(scales), n_tokens, padded, dim, out, out_dtype,
                                    out_row_stride, st);
  }
  if (scheme == ASTERQ_SCHEME_INT4 || scheme == ASTERQ_SCHEME_INT8) {
    const int dim_code = ((dim + group_size - 1) / group_size) * group_size;
    const int width = pow2_at_least(dim_code);
    if (scheme == ASTERQ_SCHEME_INT4)
      return launch_decode_d<false, 7>(width, group_size, reinterpret_cast<const uint8_t*>(codes),
                                       reinterpret_cast<const __half*>(scales), n_tokens, dim_code, dim, out, out_dtype,
                                       out_row_stride, st);
    return launch_decode_d<false, 127>(width, group_size, reinterpret_cast<const uint8_t*>(codes),
                                       reinterpret_cast<const __half*>(scales), n_tokens, dim_code, dim, out, out_dtype,
                                       out_row_stride, st);
  }
  return set_error(ASTERQ_ERR_UNSUPPORTED, "dequantize: unsupported scheme %d", scheme);
}

extern "C" int asterq_fwht(const float* x, float* y, int64_t rows, int n, void* stream) {
  clear_error();
  if (rows < 0 || n <= 0 || (n & (n - 1)))
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "fwht: length %d must be a power of two", n);
  if (rows == 0) return ASTERQ_OK;
  if (!x || !y) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "fwht: null pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (n) {
#define ASTERQ_FWHT_CASE(N)                                                                        \
  case N: {                                                                                        \
    constexpr int EPL = N < 128 ? N : 128;                                                         \
    fwht_kernel<N><<<grid_for(rows, 8 * (32 / (N / EPL))), 256, 0, st>>>(x, y, rows);              \
    return check_launch("fwht");                                                                   \
  }
    ASTERQ_FWHT_CASE(2)
    ASTERQ_FWHT_CASE(4)
    ASTERQ_FWHT_CASE(8)
    ASTERQ_FWHT_CASE(16)
    ASTERQ_FWHT_CASE(32)
    ASTERQ_FWHT_CASE(64)
    ASTERQ_FWHT_CASE(128)
    ASTERQ_FWHT_CASE(256)
    ASTERQ_FWHT_CASE(512)
#undef ASTERQ_FWHT_CASE
    default:
      return set_error(ASTERQ_ERR_UNSUPPORTED, "fwht: length %d unsupported (2..512)", n);
  }
}

extern "C" int asterq_codec_status(int32_t* timeouts) {
  clear_error();
  if (!timeouts) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "codec_status: null pointer");
  int v = 0;
  const cudaError_t e = cudaMemcpyFromSymbol(&v, g_codec_timeouts, sizeof(int));
  if (e != cudaSuccess) return set_error(ASTERQ_ERR_CUDA, "codec_status: %s", cudaGetErrorString(e));
  *timeouts = v;
  return ASTERQ_OK;
}
