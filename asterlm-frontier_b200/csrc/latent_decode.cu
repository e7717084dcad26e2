// Split-KV decode attention over the paged hybrid latent cache (sm_100a).
//
// Reference: AsterLM-Frontier src/asterlm/layers/latent_attention.py
//   _absorbed_decode :177-231  scores = (q_latent . latent + q_rope . rope) * scale,
//                              online softmax across chunks (:203-220), the new
//                              token consumed last (:226-227), ctx / max(l, 1e-20)
//   _full_attention  :116-175  q_len > 1, mask k <= past_len + i (:151-153)
// and the cache walk of src/asterlm/cache.py:139-159 (cold chunks, then hot).
//
// What the kernel computes differently from the reference (same mathematics):
//  * Cold chunks are never dequantized.  The normalized Hadamard H is symmetric
//    and orthogonal, so q . (H c) = (H q) . c: the query is rotated once per work
//    item and scored directly against the INT4 codes; the per-(token, group)
//    fp16 scale multiplies the group's partial dot product.
//  * Values of cold tokens accumulate in the rotated basis, those of hot tokens in
//    the plain basis.  One running (max, sum) covers both; the rotated accumulator
//    is rotated back once (O = H O_rot + O_plain).
//  * Tensor cores do all contractions (mma.sync m16n8k16).  Operand precision:
//    cold QK fp16 codes (exact) x rotated query split hi+lo in fp16 (per-row
//    power-of-two prescale); cold PV fp16 codes x fp16 (p * scale); hot QK bf16
//    latent x bf16 query (exact); hot PV bf16 latent x p split hi+lo in bf16.
//    Accumulation is fp32 throughout.
//
// Work decomposition: one CTA per work item = (sequence, block of 16 query rows,
// contiguous range of tiles).  Cold tiles hold 64 tokens, hot/new tiles 16.  An
// item that covers a whole sequence writes the normalized output; otherwise it
// writes an (m, l, o) partial record and combine_kernel merges the records.
//
// Warp roles (8 warps): for QK and PV warp w owns scale group w (latent dims
// 64w..64w+63); warps 0-3 also own one 16-wide slice of the RoPE dims.  QK
// partials of the 8 groups are reduced through shared memory.
#include "common.cuh"
#include "asterq_internal.h"

namespace asterq {
namespace dec {

constexpr int kL = 512;
constexpr int kRope = 64;
constexpr int kRows = 16;
constexpr int kCold = 64;
constexpr int kHot = 16;
constexpr int kThreads = 256;

// one pipeline stage
constexpr int kCodesOff = 0;                        // cold: [64][256 B] codes, 32-byte segments swizzled
constexpr int kScaleOff = kCold * 256;              // cold: [64][8] fp16 scales
constexpr int kCRopeOff = kScaleOff + kCold * 16;   // cold: [64][128 B] RoPE, 16-byte chunks swizzled
constexpr int kHotLatOff = 0;                       // hot:  [16][1024 B] latent, 16-byte chunks swizzled per 128 B
constexpr int kHotRopeOff = kHot * 1024;            // hot:  [16][128 B] RoPE
constexpr int kStageBytes = kCRopeOff + kCold * 128;  // 25600 (>= 18432 for a hot tile)

constexpr int kPartFloats = 8 * kCold * kRows;  // QK partials [warp][token][row]; also [16][512] scratch
constexpr int kRedStride = kRows + 1;
constexpr int kRedFloats = kCold * kRedStride;
constexpr int kPfColdU2 = 8 * 4 * 2 * 32;  // [group][kstep][ntile][lane] uint2 (fp16x4)
constexpr int kPfHotU2 = 2 * 2 * 32;       // [hi/lo][ntile][lane] uint2 (bf16x4)

template <int NSTAGE>
struct Smem {
  static constexpr int kStages = 0;
  static constexpr int kPart = NSTAGE * kStageBytes;
  static constexpr int kRed = kPart + kPartFloats * 4;
  static constexpr int kPfCold = kRed + kRedFloats * 4;
  static constexpr int kPfHot = kPfCold + kPfColdU2 * 8;
  static constexpr int kRowF = kPfHot + kPfHotU2 * 8;  // 6 x [16] floats
  static constexpr int kTotal = kRowF + 6 * 16 * 4;
};

// XOR swizzle of the 32-byte segments of a 256-byte code row: rows 4 apart and
// consecutive rows land in different bank octets for both access patterns.
ASTERQ_DEVICE int code_swz(int row) { return (row + (row >> 2)) & 3; }

ASTERQ_DEVICE uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
ASTERQ_DEVICE uint2 lds64(const uint8_t* p) { return *reinterpret_cast<const uint2*>(p); }

constexpr float kLog2e = 1.4426950408889634f;

// Normalized FWHT of 16 rows x 512 float32 held in shared memory (not on the
// bit-exact path: used to rotate the query and the cold accumulator).
ASTERQ_DEVICE void block_fwht16(float* buf) {
  const int tid = threadIdx.x;
#pragma unroll 1
  for (int lh = 0; lh < 9; ++lh) {
    const int h = 1 << lh;
#pragma unroll 4
    for (int b = tid; b < kRows * (kL / 2); b += kThreads) {
      const int r = b >> 8, k = b & 255;
      const int j = ((k >> lh) << (lh + 1)) | (k & (h - 1));
      float* p = buf + r * kL + j;
      const float a = p[0], c = p[h];
      p[0] = a + c;
      p[h] = a - c;
    }
    __syncthreads();
  }
  const float inv = 0.04419417382415922f;  // 1/sqrt(512)
  for (int i = tid; i < kRows * kL; i += kThreads) buf[i] *= inv;
  __syncthreads();
}

struct Tile {
  int kind, page, off, n;
};

ASTERQ_DEVICE Tile load_tile(const asterq_decode_params& p, int idx) {
  const int4 t = *reinterpret_cast<const int4*>(p.tiles + 4 * (int64_t)idx);
  Tile tile{t.x, t.y, t.z, t.w};
  // Defensive clamp: a malformed entry reads nothing instead of faulting.
  bool ok = tile.n > 0 && tile.off >= 0;
  if (tile.kind == ASTERQ_TILE_COLD) {
    ok = ok && tile.page >= 0 && tile.page < p.n_cold_pages && tile.n <= kCold && tile.off + tile.n <= p.page_tokens;
  } else if (tile.kind == ASTERQ_TILE_HOT) {
    ok = ok && tile.page >= 0 && tile.page < p.n_hot_pages && tile.n <= kHot && tile.off + tile.n <= p.page_tokens;
  } else if (tile.kind == ASTERQ_TILE_NEW) {
    ok = ok && tile.page >= 0 && tile.n <= kHot && (int64_t)tile.page + tile.off + tile.n <= p.total_q;
  } else {
    ok = false;
  }
  if (!ok) tile.n = 0;
  return tile;
}

// Issue the cp.async copies of one tile into a stage buffer.
ASTERQ_DEVICE void issue_tile(const asterq_decode_params& p, const Tile& t, uint8_t* stage) {
  const int tid = threadIdx.x;
  const uint32_t sb = smem_u32(stage);
  if (t.kind == ASTERQ_TILE_COLD) {
    const int64_t tok0 = (int64_t)t.page * p.page_tokens + t.off;
    const uint8_t* gc = reinterpret_cast<const uint8_t*>(p.cold_codes) + tok0 * 256;
    const uint8_t* gs = reinterpret_cast<const uint8_t*>(p.cold_scales) + tok0 * 16;
    const uint8_t* gr = reinterpret_cast<const uint8_t*>(p.cold_rope) + tok0 * 128;
    for (int c = tid; c < kCold * 16 + kCold + kCold * 8; c += kThreads) {
      if (c < kCold * 16) {
        const int row = c >> 4, ch = c & 15;
        if (row < t.n)
          cp_async16(sb + kCodesOff + row * 256 + (((ch >> 1) ^ code_swz(row)) << 5) + ((ch & 1) << 4),
                     gc + row * 256 + ch * 16);
      } else if (c < kCold * 17) {
        const int row = c - kCold * 16;
        if (row < t.n) cp_async16(sb + kScaleOff + row * 16, gs + row * 16);
      } else {
        const int cc = c - kCold * 17;
        const int row = cc >> 3, ch = cc & 7;
        if (row < t.n) cp_async16(sb + kCRopeOff + row * 128 + ((ch ^ (row & 7)) << 4), gr + row * 128 + ch * 16);
      }
    }
  } else {
    const uint8_t* gl;
    const uint8_t* gr;
    if (t.kind == ASTERQ_TILE_HOT) {
      const int64_t tok0 = (int64_t)t.page * p.page_tokens + t.off;
      gl = reinterpret_cast<const uint8_t*>(p.hot_latent) + tok0 * 1024;
      gr = reinterpret_cast<const uint8_t*>(p.hot_rope) + tok0 * 128;
    } else {
      const int64_t tok0 = (int64_t)t.page + t.off;
      gl = reinterpret_cast<const uint8_t*>(p.new_latent) + tok0 * 1024;
      gr = reinterpret_cast<const uint8_t*>(p.new_rope) + tok0 * 128;
    }
    for (int c = tid; c < kHot * 64 + kHot * 8; c += kThreads) {
      if (c < kHot * 64) {
        const int row = c >> 6, ch = c & 63;
        const int dst = kHotLatOff + row * 1024 + ((ch >> 3) << 7) + (((ch & 7) ^ (row & 7)) << 4);
        if (row < t.n) {
          cp_async16(sb + dst, gl + row * 1024 + ch * 16);
        } else {
          // masked value rows must be finite: P = 0 times NaN would poison the MMA
          *reinterpret_cast<uint4*>(stage + dst) = make_uint4(0u, 0u, 0u, 0u);
        }
      } else {
        const int cc = c - kHot * 64;
        const int row = cc >> 3, ch = cc & 7;
        if (row < t.n) cp_async16(sb + kHotRopeOff + row * 128 + ((ch ^ (row & 7)) << 4), gr + row * 128 + ch * 16);
      }
    }
  }
}

template <int NSTAGE>
__global__ void __launch_bounds__(kThreads, 2) decode_kernel(const asterq_decode_params p) {
  using S = Smem<NSTAGE>;
  extern __shared__ __align__(128) uint8_t smem[];
  float* spart = reinterpret_cast<float*>(smem + S::kPart);
  float* sred = reinterpret_cast<float*>(smem + S::kRed);
  uint2* pfc = reinterpret_cast<uint2*>(smem + S::kPfCold);
  uint2* pfh = reinterpret_cast<uint2*>(smem + S::kPfHot);
  float* alpha = reinterpret_cast<float*>(smem + S::kRowF);
  float* qscale = alpha + 16;
  float* qinv = alpha + 32;
  float* mrow = alpha + 48;
  float* lrow = alpha + 64;
  float* rowmax = alpha + 80;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, tq = lane & 3;
  const int* itm = p.items + 8 * (int64_t)blockIdx.x;
  const int rb = itm[1];
  // Defensive clamps: a malformed item never reads or writes out of bounds.
  const int tile_begin = max(itm[2], 0);
  const int tile_end = max(min(itm[3], p.n_tiles), tile_begin);
  const int slot = (itm[4] < p.n_slots) ? itm[4] : -2;  // -2: out-of-range slot, write nothing
  const int64_t out_row0 = itm[5];
  const int n_rows = min(itm[6], kRows);
  const int H = p.n_heads;

  // ---------------- prologue: rotated, prescaled query fragments ----------------
  {
    const uint16_t* ql = reinterpret_cast<const uint16_t*>(p.q_lat);
    for (int i = tid; i < kRows * kL / 8; i += kThreads) {
      const int r = i >> 6, c8 = i & 63;
      uint4 w = make_uint4(0u, 0u, 0u, 0u);
      if (r < n_rows) w = *reinterpret_cast<const uint4*>(ql + (out_row0 + r) * kL + 8 * c8);
      float* d = spart + r * kL + 8 * c8;
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        d[2 * k] = bf16lo_to_f32(ws[k]);
        d[2 * k + 1] = bf16hi_to_f32(ws[k]);
      }
    }
    __syncthreads();
    block_fwht16(spart);
    {
      const int r = tid >> 4, part = tid & 15;
      float mx = 0.0f;
      for (int k = 0; k < 32; ++k) mx = fmaxf(mx, fabsf(spart[r * kL + 32 * part + k]));
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      if (part == 0) rowmax[r] = mx;
    }
    __syncthreads();
    if (tid < kRows) {
      const float mx = rowmax[tid];
      int e = 0;
      if (mx > 0.0f) {
        int ex;
        frexpf(mx, &ex);
        e = min(max(14 - ex, -100), 100);
      }
      qscale[tid] = ldexpf(1.0f, e);
      qinv[tid] = ldexpf(1.0f, -e) * p.softmax_scale;
    }
    __syncthreads();
  }

  uint32_t qc[4][2][2][2];  // cold: [kstep][ntile][hi/lo][b0/b1] fp16, K-permuted to match the code layout
  uint32_t qh[4][2][2];     // hot:  [kstep][ntile][b0/b1] bf16
  uint32_t qr[2][2];        // rope: [ntile][b0/b1] bf16 (warps 0-3)
  {
    const uint16_t* ql = reinterpret_cast<const uint16_t*>(p.q_lat);
    const uint16_t* qrp = reinterpret_cast<const uint16_t*>(p.q_rope);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int row = 8 * nt + gid;
      const float sc = qscale[row];
      const bool rv = row < n_rows;
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        // K permutation: see the code-fragment extraction in the cold QK loop
        const int base = 64 * warp + 16 * tq + 8 * (s >> 1) + 2 * (s & 1);
        const int dims[4] = {base, base + 4, base + 1, base + 5};
        float x[4];
        __half hi[4], lo[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          x[k] = spart[row * kL + dims[k]] * sc;
          hi[k] = __float2half_rn(x[k]);
          lo[k] = __float2half_rn(x[k] - __half2float(hi[k]));
        }
        qc[s][nt][0][0] = (uint32_t)__half_as_ushort(hi[0]) | ((uint32_t)__half_as_ushort(hi[1]) << 16);
        qc[s][nt][0][1] = (uint32_t)__half_as_ushort(hi[2]) | ((uint32_t)__half_as_ushort(hi[3]) << 16);
        qc[s][nt][1][0] = (uint32_t)__half_as_ushort(lo[0]) | ((uint32_t)__half_as_ushort(lo[1]) << 16);
        qc[s][nt][1][1] = (uint32_t)__half_as_ushort(lo[2]) | ((uint32_t)__half_as_ushort(lo[3]) << 16);
        // hot query: plain basis, bf16 (exact after the power-of-two prescale)
        const int e0 = 64 * warp + 16 * s + 2 * tq;
        uint32_t w0 = 0u, w1 = 0u;
        if (rv) {
          w0 = *reinterpret_cast<const uint32_t*>(ql + (out_row0 + row) * kL + e0);
          w1 = *reinterpret_cast<const uint32_t*>(ql + (out_row0 + row) * kL + e0 + 8);
        }
        const float2 f0 = unpack_bf162(w0), f1 = unpack_bf162(w1);
        qh[s][nt][0] = pack_bf162(f0.x * sc, f0.y * sc);
        qh[s][nt][1] = pack_bf162(f1.x * sc, f1.y * sc);
      }
      uint32_t r0 = 0u, r1 = 0u;
      if (rv && warp < 4) {
        const int e0 = 16 * warp + 2 * tq;
        r0 = *reinterpret_cast<const uint32_t*>(qrp + (out_row0 + row) * kRope + e0);
        r1 = *reinterpret_cast<const uint32_t*>(qrp + (out_row0 + row) * kRope + e0 + 8);
      }
      const float2 g0 = unpack_bf162(r0), g1 = unpack_bf162(r1);
      qr[nt][0] = pack_bf162(g0.x * sc, g0.y * sc);
      qr[nt][1] = pack_bf162(g1.x * sc, g1.y * sc);
    }
  }
  __syncthreads();  // spart is reused below

  // ---------------- main loop over tiles ----------------
  float o[4][2][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int k = 0; k < 4; ++k) o[i][j][k] = 0.0f;

  const int n_t = tile_end - tile_begin;
  // order 0: accumulator holds cold tokens, rotated basis, code-derived row order
  // order 1: plain basis, natural row order
  int order = 0;
  if (n_t > 0) {
    const int k0 = p.tiles[4 * (int64_t)tile_begin];  // tile_begin < tile_end <= n_tiles
    order = (k0 == ASTERQ_TILE_COLD) ? 0 : 1;
  }
  float m_run = -INFINITY, l_run = 0.0f;  // softmax state of row tid>>4 (replicated over 16 threads)
  const int srow = tid >> 4, sj = tid & 15;

#pragma unroll 1
  for (int i = 0; i < NSTAGE - 1; ++i) {
    if (i < n_t) issue_tile(p, load_tile(p, tile_begin + i), smem + i * kStageBytes);
    cp_async_commit();
  }

#pragma unroll 1
  for (int ti = 0; ti < n_t; ++ti) {
    {
      const int nxt = ti + NSTAGE - 1;
      if (nxt < n_t) issue_tile(p, load_tile(p, tile_begin + nxt), smem + (nxt % NSTAGE) * kStageBytes);
      cp_async_commit();
    }
    const Tile t = load_tile(p, tile_begin + ti);
    const uint8_t* st = smem + (ti % NSTAGE) * kStageBytes;
    cp_async_wait<NSTAGE - 1>();
    __syncthreads();

    const bool cold = (t.kind == ASTERQ_TILE_COLD);
    // ---------------- QK: per-warp partial scores ----------------
    if (cold) {
#pragma unroll 1
      for (int m = 0; m < 4; ++m) {
        float acc[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int k = 0; k < 4; ++k) acc[j][k] = 0.0f;
        const int r0 = 16 * m + gid, r1 = r0 + 8;
        const uint2 v0 = lds64(st + kCodesOff + r0 * 256 + ((warp ^ code_swz(r0)) << 5) + 8 * tq);
        const uint2 v1 = lds64(st + kCodesOff + r1 * 256 + ((warp ^ code_swz(r1)) << 5) + 8 * tq);
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          // word w covers dims 16tq + 8w + j (nibble j); k-step s uses word s>>1,
          // nibble pairs (0,4),(1,5) for even s and (2,6),(3,7) for odd s.
          uint32_t x0 = (s < 2) ? v0.x : v0.y;
          uint32_t x1 = (s < 2) ? v1.x : v1.y;
          if (s & 1) {
            x0 >>= 8;
            x1 >>= 8;
          }
          uint32_t a[4];
          a[0] = nib_lo_f16x2(x0);
          a[1] = nib_lo_f16x2(x1);
          a[2] = nib_hi_f16x2(x0);
          a[3] = nib_hi_f16x2(x1);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            mma_f16(acc[nt], a, qc[s][nt][0][0], qc[s][nt][0][1]);
            mma_f16(acc[nt], a, qc[s][nt][1][0], qc[s][nt][1][1]);
          }
        }
        const __half* scl = reinterpret_cast<const __half*>(st + kScaleOff);
        const float s0 = __half2float(scl[r0 * 8 + warp]);
        const float s1 = __half2float(scl[r1 * 8 + warp]);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          acc[nt][0] *= s0;
          acc[nt][1] *= s0;
          acc[nt][2] *= s1;
          acc[nt][3] *= s1;
        }
        if (warp < 4) {
          const int row = 16 * m + (lane & 7) + 8 * ((lane >> 3) & 1);
          const int ch = 2 * warp + (lane >> 4);
          uint32_t ra[4];
          ldmatrix_x4(ra, smem_u32(st + kCRopeOff + row * 128 + ((ch ^ (row & 7)) << 4)));
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) mma_bf16(acc[nt], ra, qr[nt][0], qr[nt][1]);
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          *reinterpret_cast<float2*>(spart + (warp * kCold + r0) * kRows + 8 * nt + 2 * tq) =
              make_float2(acc[nt][0], acc[nt][1]);
          *reinterpret_cast<float2*>(spart + (warp * kCold + r1) * kRows + 8 * nt + 2 * tq) =
              make_float2(acc[nt][2], acc[nt][3]);
        }
      }
    } else {
      float acc[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[j][k] = 0.0f;
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const int row = (lane & 7) + 8 * ((lane >> 3) & 1);
        const int ch = 2 * s + (lane >> 4);
        uint32_t a[4];
        ldmatrix_x4(a, smem_u32(st + kHotLatOff + row * 1024 + (warp << 7) + ((ch ^ (row & 7)) << 4)));
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) mma_bf16(acc[nt], a, qh[s][nt][0], qh[s][nt][1]);
      }
      if (warp < 4) {
        const int row = (lane & 7) + 8 * ((lane >> 3) & 1);
        const int ch = 2 * warp + (lane >> 4);
        uint32_t ra[4];
        ldmatrix_x4(ra, smem_u32(st + kHotRopeOff + row * 128 + ((ch ^ (row & 7)) << 4)));
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) mma_bf16(acc[nt], ra, qr[nt][0], qr[nt][1]);
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        *reinterpret_cast<float2*>(spart + (warp * kCold + gid) * kRows + 8 * nt + 2 * tq) =
            make_float2(acc[nt][0], acc[nt][1]);
        *reinterpret_cast<float2*>(spart + (warp * kCold + gid + 8) * kRows + 8 * nt + 2 * tq) =
            make_float2(acc[nt][2], acc[nt][3]);
      }
    }
    __syncthreads();

    // ---------------- reduce the 8 group partials, scale, mask ----------------
    const int ntok = cold ? kCold : kHot;
    {
      const int tok = tid >> 2, rq = tid & 3;
      if (tok < ntok) {
        float4 acc = *reinterpret_cast<const float4*>(spart + tok * kRows + 4 * rq);
#pragma unroll
        for (int w = 1; w < 8; ++w) {
          const float4 v = *reinterpret_cast<const float4*>(spart + (w * kCold + tok) * kRows + 4 * rq);
          acc.x += v.x;
          acc.y += v.y;
          acc.z += v.z;
          acc.w += v.w;
        }
        const float vals[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int r = 4 * rq + c;
          float sv = vals[c] * qinv[r];
          if (p.logit_softcap > 0.0f) sv = p.logit_softcap * tanhf(sv / p.logit_softcap);
          bool valid = tok < t.n;
          if (t.kind == ASTERQ_TILE_NEW) valid = valid && (t.off + tok) <= (rb * kRows + r) / H;
          sred[tok * kRedStride + r] = valid ? sv : -INFINITY;
        }
      }
    }
    __syncthreads();

    // ---------------- online softmax (latent_attention.py:203-220) ----------------
    {
      float sv[4];
      float tmax = -INFINITY;
      if (cold) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          sv[i] = sred[(4 * sj + i) * kRedStride + srow];
          tmax = fmaxf(tmax, sv[i]);
        }
      } else {
        sv[0] = sred[sj * kRedStride + srow];
        sv[1] = sv[2] = sv[3] = -INFINITY;
        tmax = sv[0];
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
      const float m_new = fmaxf(m_run, tmax);
      float a_r, msub;
      if (m_new == -INFINITY) {
        a_r = 1.0f;
        msub = 0.0f;
      } else {
        a_r = exp2f((m_run - m_new) * kLog2e);
        msub = m_new;
      }
      float pv[4];
      float psum = 0.0f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        pv[i] = exp2f((sv[i] - msub) * kLog2e);
        psum += pv[i];
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
      l_run = l_run * a_r + psum;
      m_run = m_new;
      if (sj == 0) alpha[srow] = a_r;
      if (cold) {
        const uint8_t* scl = st + kScaleOff;
        uint4 sc[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) sc[i] = *reinterpret_cast<const uint4*>(scl + (4 * sj + i) * 16);
        const int kt = sj >> 2, nt = srow >> 3;
        const int ln = (srow & 7) * 4 + (sj & 3);
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          float f[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t wd = (&sc[i].x)[g >> 1];
            const float s = (g & 1) ? unpack_half2(wd).y : unpack_half2(wd).x;
            f[i] = (4 * sj + i < t.n) ? pv[i] * s : 0.0f;
          }
          pfc[((g * 4 + kt) * 2 + nt) * 32 + ln] = make_uint2(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]));
        }
      } else {
        const float pp = pv[0];
        const __nv_bfloat16 hi = __float2bfloat16_rn(pp);
        const __nv_bfloat16 lo = __float2bfloat16_rn(pp - __bfloat162float(hi));
        const int nt = srow >> 3;
        const int ln = (srow & 7) * 4 + ((sj & 7) >> 1);
        uint16_t* ph = reinterpret_cast<uint16_t*>(pfh);
        const int idx = (sj >> 3) * 2 + (sj & 1);
        ph[((0 * 2 + nt) * 32 + ln) * 4 + idx] = __bfloat16_as_ushort(hi);
        ph[((1 * 2 + nt) * 32 + ln) * 4 + idx] = __bfloat16_as_ushort(lo);
      }
    }
    __syncthreads();

    // ---------------- basis change before the first hot tile ----------------
    if (!cold && order == 0) {
#pragma unroll
      for (int mi = 0; mi < 4; ++mi)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int dim = 64 * warp + 2 * (4 * gid + mi) + (c >> 1);
            const int row = 8 * nt + 2 * tq + (c & 1);
            spart[row * kL + dim] = o[mi][nt][c];
          }
      __syncthreads();
      block_fwht16(spart);
#pragma unroll
      for (int mi = 0; mi < 4; ++mi)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int dim = 64 * warp + 16 * mi + gid + 8 * (c >> 1);
            const int row = 8 * nt + 2 * tq + (c & 1);
            o[mi][nt][c] = spart[row * kL + dim];
          }
      order = 1;
      __syncthreads();
    }

    // ---------------- PV ----------------
    {
      float al[2][2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        al[nt][0] = alpha[8 * nt + 2 * tq];
        al[nt][1] = alpha[8 * nt + 2 * tq + 1];
      }
#pragma unroll
      for (int mi = 0; mi < 4; ++mi)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          o[mi][nt][0] *= al[nt][0];
          o[mi][nt][1] *= al[nt][1];
          o[mi][nt][2] *= al[nt][0];
          o[mi][nt][3] *= al[nt][1];
        }
    }
    if (cold) {
#pragma unroll 1
      for (int kt = 0; kt < 4; ++kt) {
        uint32_t x[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = 16 * kt + 4 * tq + i;
          x[i] = lds32(st + kCodesOff + row * 256 + ((warp ^ code_swz(row)) << 5) + 4 * gid);
        }
        uint2 pb[2];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) pb[nt] = pfc[((warp * 4 + kt) * 2 + nt) * 32 + lane];
#pragma unroll
        for (int mi = 0; mi < 4; ++mi) {
          // rows gid / gid+8 of m-tile mi are dims 2(4gid+mi) / 2(4gid+mi)+1 (the two
          // nibbles of byte 4gid+mi); columns k are tokens 4tq+{0,1} / 4tq+{2,3}
          const uint32_t sel = (uint32_t)mi | ((uint32_t)mi << 4) | ((uint32_t)(4 + mi) << 8) | ((uint32_t)(4 + mi) << 12);
          const uint32_t z01 = prmt(x[0], x[1], sel);
          const uint32_t z23 = prmt(x[2], x[3], sel);
          uint32_t a[4];
          a[0] = nib_lo_f16x2(z01);
          a[1] = nib_hi_f16x2(z01);
          a[2] = nib_lo_f16x2(z23);
          a[3] = nib_hi_f16x2(z23);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) mma_f16(o[mi][nt], a, pb[nt].x, pb[nt].y);
        }
      }
    } else {
#pragma unroll
      for (int mi = 0; mi < 4; ++mi) {
        const int row = (lane & 7) + 8 * (lane >> 4);
        const int ch = 2 * mi + ((lane >> 3) & 1);
        uint32_t a[4];
        ldmatrix_x4_trans(a, smem_u32(st + kHotLatOff + row * 1024 + (warp << 7) + ((ch ^ (row & 7)) << 4)));
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
          for (int hl = 0; hl < 2; ++hl) {
            const uint2 b = pfh[(hl * 2 + nt) * 32 + lane];
            mma_bf16(o[mi][nt], a, b.x, b.y);
          }
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // ---------------- epilogue ----------------
  if (sj == 0) {
    mrow[srow] = m_run;
    lrow[srow] = l_run;
  }
#pragma unroll
  for (int mi = 0; mi < 4; ++mi)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int dim = (order == 0) ? 64 * warp + 2 * (4 * gid + mi) + (c >> 1) : 64 * warp + 16 * mi + gid + 8 * (c >> 1);
        const int row = 8 * nt + 2 * tq + (c & 1);
        spart[row * kL + dim] = o[mi][nt][c];
      }
  __syncthreads();
  if (order == 0) block_fwht16(spart);

  if (slot == -1) {
    for (int i = tid; i < kRows * kL / 4; i += kThreads) {
      const int r = i >> 7, c4 = i & 127;
      if (r >= n_rows) continue;
      const float inv = 1.0f / fmaxf(lrow[r], 1e-20f);
      const float4 v = *reinterpret_cast<const float4*>(spart + r * kL + 4 * c4);
      const int64_t off = (out_row0 + r) * kL + 4 * c4;
      if (p.out_dtype == ASTERQ_DTYPE_F32) {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + off) =
            make_float4(v.x * inv, v.y * inv, v.z * inv, v.w * inv);
      } else {
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.out) + off) =
            make_uint2(pack_bf162(v.x * inv, v.y * inv), pack_bf162(v.z * inv, v.w * inv));
      }
    }
  } else if (slot >= 0) {
    float* wo = reinterpret_cast<float*>(p.workspace);
    float* wm = wo + (int64_t)p.n_slots * kRows * kL;
    float* wl = wm + (int64_t)p.n_slots * kRows;
    for (int i = tid; i < kRows * kL / 4; i += kThreads) {
      const int r = i >> 7, c4 = i & 127;
      *reinterpret_cast<float4*>(wo + ((int64_t)slot * kRows + r) * kL + 4 * c4) =
          *reinterpret_cast<const float4*>(spart + r * kL + 4 * c4);
    }
    if (tid < kRows) {
      wm[(int64_t)slot * kRows + tid] = mrow[tid];
      wl[(int64_t)slot * kRows + tid] = lrow[tid];
    }
  }
}

// Merge partial records (latent_attention.py:212-220 applied across splits).
// Grid: (combine job, 32-dim slice of the latent); 256 threads = 16 rows x 16
// pairs of dims, so a long sequence's many records are read by many CTAs.
constexpr int kCombDims = 32;
__global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ wo, const float* __restrict__ wm,
                                                      const float* __restrict__ wl, const int32_t* __restrict__ jobs,
                                                      int n_slots, int latent_dim, void* __restrict__ out,
                                                      int out_dtype) {
  const int4 job = *reinterpret_cast<const int4*>(jobs + 4 * (int64_t)blockIdx.x);
  const int slot_begin = max(job.x, 0), slot_end = min(job.y, n_slots), n_rows = min(job.w, kRows);
  const int64_t out_row0 = job.z;
  const int r = threadIdx.x >> 4, d = blockIdx.y * kCombDims + 2 * (threadIdx.x & 15);
  if (r >= n_rows || slot_end <= slot_begin || d >= latent_dim) return;
  float mmax = -INFINITY;
  for (int s = slot_begin; s < slot_end; ++s) mmax = fmaxf(mmax, wm[(int64_t)s * kRows + r]);
  const float msub = (mmax == -INFINITY) ? 0.0f : mmax;
  float l = 0.0f, a0 = 0.0f, a1 = 0.0f;
  for (int s = slot_begin; s < slot_end; ++s) {
    const float w = exp2f((wm[(int64_t)s * kRows + r] - msub) * kLog2e);
    l += w * wl[(int64_t)s * kRows + r];
    const float2 v = *reinterpret_cast<const float2*>(wo + ((int64_t)s * kRows + r) * latent_dim + d);
    a0 += w * v.x;
    a1 += w * v.y;
  }
  const float inv = 1.0f / fmaxf(l, 1e-20f);
  const int64_t off = (out_row0 + r) * latent_dim + d;
  if (out_dtype == ASTERQ_DTYPE_F32) {
    *reinterpret_cast<float2*>(reinterpret_cast<float*>(out) + off) = make_float2(a0 * inv, a1 * inv);
  } else {
    *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(out) + off) = pack_bf162(a0 * inv, a1 * inv);
  }
}

constexpr int kNStage = 2;

int validate(const asterq_decode_params* p) {
  if (!p) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: null params");
  if (p->latent_dim != kL || p->rope_dim != kRope || p->group_size != 64)
    return set_error(ASTERQ_ERR_UNSUPPORTED, "decode: geometry latent=%d rope=%d group=%d unsupported (512/64/64)",
                     p->latent_dim, p->rope_dim, p->group_size);
  if (p->n_heads <= 0) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: n_heads must be positive");
  if (p->page_tokens <= 0 || p->page_tokens % kCold)
    return set_error(ASTERQ_ERR_UNSUPPORTED, "decode: page_tokens %d must be a positive multiple of %d",
                     p->page_tokens, kCold);
  if (p->out_dtype != ASTERQ_DTYPE_F32 && p->out_dtype != ASTERQ_DTYPE_BF16)
    return set_error(ASTERQ_ERR_UNSUPPORTED, "decode: out_dtype must be f32 or bf16");
  if (p->n_items < 0 || p->n_tiles < 0 || p->n_combine < 0 || p->n_slots < 0)
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: negative table size");
  if (p->n_items > 0 && (!p->items || !p->tiles || !p->q_lat || !p->q_rope || !p->out))
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: null pointer");
  if (p->n_cold_pages > 0 && (!p->cold_codes || !p->cold_scales || !p->cold_rope))
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: null cold pool");
  if (p->n_hot_pages > 0 && (!p->hot_latent || !p->hot_rope))
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: null hot pool");
  const void* aligned[] = {p->q_lat, p->q_rope, p->new_latent, p->new_rope, p->cold_codes, p->cold_scales,
                           p->cold_rope, p->hot_latent, p->hot_rope, p->tiles, p->items, p->combine, p->out,
                           p->workspace};
  for (const void* ptr : aligned)
    if (reinterpret_cast<uintptr_t>(ptr) & 15) return set_error(ASTERQ_ERR_MISALIGNED, "decode: pointers must be 16-byte aligned");
  const int64_t need = (int64_t)p->n_slots * kRows * (kL + 2) * 4;
  if (p->n_slots > 0 && (!p->workspace || p->workspace_bytes < need))
    return set_error(ASTERQ_ERR_WORKSPACE, "decode: workspace of %lld bytes < %lld needed",
                     (long long)p->workspace_bytes, (long long)need);
  return ASTERQ_OK;
}

}  // namespace dec
}  // namespace asterq

using namespace asterq;

extern "C" int64_t asterq_decode_workspace_bytes(const asterq_decode_params* p) {
  if (!p || p->n_slots <= 0) return 0;
  return (int64_t)p->n_slots * dec::kRows * (dec::kL + 2) * 4;
}

extern "C" int asterq_latent_decode(const asterq_decode_params* p, void* stream) {
  clear_error();
  int st = dec::validate(p);
  if (st != ASTERQ_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  using S = dec::Smem<dec::kNStage>;
  if (p->n_items > 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    static unsigned long long configured = 0;  // one bit per device ordinal
    if (dev >= 64 || !(configured & (1ull << dev))) {
      cudaError_t e = cudaFuncSetAttribute(dec::decode_kernel<dec::kNStage>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal);
      if (e != cudaSuccess) return set_error(ASTERQ_ERR_CUDA, "latent_decode: %s", cudaGetErrorString(e));
      if (dev < 64) configured |= (1ull << dev);
    }
    dec::decode_kernel<dec::kNStage><<<p->n_items, dec::kThreads, S::kTotal, s>>>(*p);
    st = check_launch("latent_decode");
    if (st != ASTERQ_OK) return st;
  }
  if (p->n_combine > 0) {
    const float* wo = reinterpret_cast<const float*>(p->workspace);
    const float* wm = wo + (int64_t)p->n_slots * dec::kRows * dec::kL;
    const float* wl = wm + (int64_t)p->n_slots * dec::kRows;
    dec::combine_kernel<<<dim3(p->n_combine, dec::kL / dec::kCombDims), 256, 0, s>>>(wo, wm, wl, p->combine, p->n_slots, dec::kL, p->out,
                                                     p->out_dtype);
    st = check_launch("splitkv_combine");
  }
  return st;
}

extern "C" int asterq_splitkv_combine(const float* partials, int32_t n_slots, const int32_t* combine,
                                      int32_t n_combine, int32_t latent_dim, void* out, int32_t out_dtype,
                                      void* stream) {
  clear_error();
  if (latent_dim != dec::kL) return set_error(ASTERQ_ERR_UNSUPPORTED, "combine: latent_dim must be 512");
  if (n_slots < 0 || n_combine < 0) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "combine: negative sizes");
  if (n_combine == 0) return ASTERQ_OK;
  if (!partials || !combine || !out) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "combine: null pointer");
  if (out_dtype != ASTERQ_DTYPE_F32 && out_dtype != ASTERQ_DTYPE_BF16)
    return set_error(ASTERQ_ERR_UNSUPPORTED, "combine: out_dtype must be f32 or bf16");
  if ((reinterpret_cast<uintptr_t>(partials) | reinterpret_cast<uintptr_t>(combine) | reinterpret_cast<uintptr_t>(out)) & 15)
    return set_error(ASTERQ_ERR_MISALIGNED, "combine: pointers must be 16-byte aligned");
  const float* wm = partials + (int64_t)n_slots * dec::kRows * latent_dim;
  const float* wl = wm + (int64_t)n_slots * dec::kRows;
  dec::combine_kernel<<<dim3(n_combine, dec::kL / dec::kCombDims), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(partials, wm, wl, combine, n_slots,
                                                                                     latent_dim, out, out_dtype);
  return check_launch("splitkv_combine");
}
