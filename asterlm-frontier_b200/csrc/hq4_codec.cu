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
  if (!x || !codes || !scales) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "quantize: null pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (scheme == ASTERQ_SCHEME_HADAMARD_INT4) {
    const int padded = pow2_at_least(dim);
    if (padded % group_size) return set_error(ASTERQ_ERR_UNSUPPORTED, "quantize: group %d does not divide %d", group_size, padded);
    if ((reinterpret_cast<uintptr_t>(codes) & 15) || (reinterpret_cast<uintptr_t>(scales) & 1))
      return set_error(ASTERQ_ERR_MISALIGNED, "quantize: codes must be 16-byte aligned");
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
  if (!codes || !scales || !out) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "dequantize: null pointer");
  if (out_dtype != ASTERQ_DTYPE_F32 && out_dtype != ASTERQ_DTYPE_BF16 && out_dtype != ASTERQ_DTYPE_F16)
    return set_error(ASTERQ_ERR_UNSUPPORTED, "dequantize: unsupported output dtype %d", out_dtype);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
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
