// Split-KV decode attention over the paged hybrid latent cache (sm_100a).
//
// Reference: AsterLM-Frontier src/asterlm/layers/latent_attention.py
//   _absorbed_decode :177-231  scores = (q_latent . latent + q_rope . rope) * scale,
//                              online softmax across chunks (:203-220), the new
//                              token consumed last (:226-227), ctx / max(l, 1e-20)
//   _full_attention  :116-175  q_len > 1, mask k <= past_len + i (:151-153)
// and the cache walk of src/asterlm/cache.py:139-159 (cold chunks, then hot).
//
// Same mathematics, computed differently:
//  * Cold chunks are never dequantized to memory.  The normalized Hadamard H is
//    symmetric and orthogonal, so q . (H c) = (H q) . c: the query is rotated once
//    per work item and scored directly against the INT4 codes; the per-(token,
//    group) fp16 scale multiplies the group's partial dot product.
//  * Values of cold tokens accumulate in the rotated basis, those of hot tokens in
//    the plain basis, under one running (max, sum); the rotated accumulator is
//    rotated back once (O = H O_rot + O_plain).
//  * Tensor-core operands: cold QK runs on the int8 tensor path (m16n8k32): the
//    codes expand to exact signed bytes (16 x code, two logic ops per four
//    values) and the rotated query is a per-row 16-bit fixed-point number split
//    into two int8 limbs; each scale group's integer dot products start from a
//    float-exponent bias so that the int32 accumulator reads as an exact fp32
//    value, then scale x (256 hi + lo) is accumulated in fp32.  Cold PV = fp16
//    codes x fp16 p times the fp16 code scale; hot QK = bf16 latent x bf16
//    query (exact); hot PV = bf16 latent x p split hi + lo in bf16; RoPE = bf16
//    x bf16; fp32 accumulation everywhere.
//
// CTA organisation (one CTA per work item, 16 warps):
//  * TMA producer (lane 0 of warp 8): streams the item's tiles (128 cold tokens or
//    32 hot/new tokens) into a 3-stage ring with cp.async.bulk.tensor (128-byte
//    hardware swizzle) and mbarrier completion; tile i+3 is issued as soon as
//    tile i's team and the value warps have released it.
//  * warps 0-7 ("score warps"): two teams of 4 that take alternate tiles, so one
//    team's softmax overlaps the other's QK.  In a team each warp owns a quarter of
//    the tile's tokens and all 512 latent dims, so every score row is complete
//    inside one warp.  The team finishes the online softmax (one named barrier per
//    team for the tile maxima; the running max passes between the teams) and hands
//    p to the value warps through shared memory, one buffer per team (cold tiles:
//    fp16 [token][row] plus the tokens' code scales by group; hot tiles: fp32
//    [row][token]).
//  * warps 8-15 ("value warps"): each owns 64 latent dims (one scale group) of
//    the 16 x 512 accumulator and accumulates p . V for every tile, in order.
// setmaxnreg gives the score warpgroups 160 registers and the value warpgroups 96.
// Every wait is bounded; a timeout sets a status flag instead of hanging.
#include <atomic>
#include <mutex>
#include <string.h>
#include <cuda.h>

#include "common.cuh"
#include "asterq_internal.h"

namespace asterq {
namespace dec {

constexpr int kL = 512;
constexpr int kRope = 64;
constexpr int kRows = 16;
constexpr int kColdTile = 128;
constexpr int kColdTile8 = 64;     // int8 codes: tokens of a cold tile
constexpr int kCodeBlock8 = 8192;  // int8 codes: dims 128b..128b+127 of the tile's 64 tokens at b * 8192, SW128
constexpr int kHotTile = 32;
constexpr int kStages = 3;
constexpr int kTeamWarps = 4;                  // score warps of one team (one tile at a time)
constexpr int kScoreWarps = 2 * kTeamWarps;    // two teams take alternate tiles
constexpr int kValueWarps = 8;
constexpr int kProducerWarp = kScoreWarps;     // lane 0 of the first value warp issues the TMA loads
constexpr int kThreads = 32 * (kScoreWarps + kValueWarps);
// Register split (setmaxnreg; the launch gives every thread 128): score warps hold two
// groups of int8 accumulators in flight, value warps one 16 x 64 fp32 accumulator.
constexpr int kScoreRegs = 160;
constexpr int kValueRegs = 96;
constexpr int kLaunchRegs = 128;
// the one-byte-code modes: one m-tile per score warp needs fewer score registers, and their value
// warps' code bytes need more (at 96 they spill)
constexpr int kScoreRegsB = 144;
constexpr int kValueRegsB = 112;
static_assert(32 * (kScoreWarps * kScoreRegsB + kValueWarps * kValueRegsB) <= kThreads * kLaunchRegs,
              "setmaxnreg split of the byte-code modes exceeds the launch's register allocation");
static_assert(32 * (kScoreWarps * kScoreRegs + kValueWarps * kValueRegs) <= kThreads * kLaunchRegs,
              "setmaxnreg split exceeds the launch's register allocation");

// one pipeline stage (offsets in bytes, swizzled regions 1024-aligned)
constexpr int kCodesLo = 0;        // cold: [128][128 B] codes of dims 0..255, SW128
constexpr int kCodesHi = 16384;    // cold: [128][128 B] codes of dims 256..511, SW128
constexpr int kCRope = 32768;      // cold: [128][128 B] RoPE keys, SW128; quantized RoPE (ASTERQ_ROPE_QUANTIZED):
                                   // [128][32 B] codes, plain
constexpr int kCRopeScale = kCRope + 4096;  // quantized RoPE: fp16 scales of the tile's tokens from the
                                            // 8-token boundary at or below its first token
constexpr int kScales = 49152;     // cold: [128][16 B] fp16 scales, plain
constexpr int kHotBlock = 4096;    // hot: latent scale-group g at g*4096: [32][128 B], SW128
constexpr int kHRope = 32768;      // hot: [32][128 B] RoPE keys, SW128
constexpr int kHotPartial = 36864; // hot, byte-code modes: the score team's partial scores
constexpr int kPartStride = 20;    //   [4 warps][32 tokens][kPartStride floats] (padded row stride)
constexpr int kStageBytes = 51200;
static_assert(kHotPartial + 4 * 32 * kPartStride * 4 <= kStageBytes, "hot partial scores fit the stage's tail");

constexpr int kOffQi = kStages * kStageBytes;  // cold query int8 limb fragments [16 k-steps][2][32] uint4
                                               // (32 KB region: the [16][512] fp32 scratch after the tiles)
constexpr int kOffQri = kOffQi + 16384;         // quantized RoPE: query int8 limb fragments [2][2][32] uint4
                                                // (in the scratch half that the tile loop leaves unused)
constexpr int kOffQh = kOffQi + 32768;          // hot query B fragments  [8][4][2][32] uint2
constexpr int kOffQr = kOffQh + 16384;          // rope query B fragments [4][2][32] uint2
constexpr int kPStride = kColdTile + 4;         // p tile row stride (floats)
constexpr int kPBytes = kRows * kPStride * 4;
constexpr int kOffP = kOffQr + 2048;            // 2 x p tile [16][132] fp32
constexpr int kOffST = kOffP + 2 * kPBytes;     // 2 x cold code scales [8 groups][128 tokens] fp16
constexpr int kOffMisc = kOffST + 2 * 2048;     // 1024 floats of per-row scalars
constexpr int kOffBar = kOffMisc + 4096;        // mbarriers
constexpr int kSmemBytes = kOffBar + 192 + 1024;  // + alignment slack
static_assert(kSmemBytes <= 232448, "dynamic shared memory per block");

// misc (float index)
constexpr int kMAlpha = 0;     // [2][16]
constexpr int kMQscale = 32;   // [16]
constexpr int kMQinv = 48;     // [16]  (score multiplier 2^-e * softmax_scale)
constexpr int kMQint = 64;     // [16]  fixed-point query scale (32511 / max |rotated row|)
constexpr int kMQinvI = 80;    // [16]  cold integer-score multiplier softmax_scale / (16 * kMQint)
constexpr int kMRopeR = 96;    // [16]  RoPE score -> integer-score units (kMQinv / kMQinvI); with quantized
                               //       RoPE keys: kMQint / (the RoPE query's own fixed-point scale)
constexpr int kQScalars = 80;  // kMQscale .. kMRopeR: the per-row scalars of a prepared query block
constexpr int kMWmax = 112;    // [2 teams][2][4][16] tile maxima (a team's tiles alternate buffers);
                               // after the tile loop [16] = final running max
constexpr int kMLw = 368;      // [8 score warps][16]
constexpr int kMMrun = 496;    // [2][16] running max after tile i, in slot i & 1 (team hand-off)
constexpr int kMComb = 528;    // fused combine: [2][16] per-row max and 1 / sum, then [8][16] part weights

// workspace: n_slots partial records, then n_units prepared query blocks
constexpr int kRecordBytes = kRows * (kL + 2) * 4;                    // 32,896
constexpr int kQPrepRopeInt = 16384 + 16384 + 2048 + 512;             // quantized RoPE limb fragments
constexpr int kQPrepBytes = kQPrepRopeInt + 2048;                     // 37,376: qi | qh | qr | scalars | qri
// then one int32 per unit: partial records written so far (fused combine jobs)
__host__ __device__ inline int64_t counters_offset(int n_slots, int n_units) {
  return (int64_t)n_slots * kRecordBytes + (int64_t)n_units * kQPrepBytes;
}
inline int64_t counter_bytes(int n_units) { return ((int64_t)n_units * 4 + 15) / 16 * 16; }
constexpr uint32_t kQPrepCopyBytes = 16384 + 16384 + 2048 + 4 * kQScalars;

// mbarrier slots (8 bytes each)
// Tile i lands in stage i % 3 and completes barrier kBarFull + i % 6: each of those six
// barriers serves one team's tiles only (i and i + 6 have the same parity), so a team's
// parity wait on it is never one phase behind or ahead of the tile it wants.
constexpr int kFullBars = 2 * kStages;
constexpr int kBarFull = 0;    // [6] TMA landed
constexpr int kBarEmpty = 6;   // [3] the tile's team + value warps done with a stage
constexpr int kBarPFull = 9;   // [2] p tile written
constexpr int kBarPEmpty = 11; // [2] p tile consumed
constexpr int kBarAbort = 13;  // int flag (shares the slot area)
constexpr int kBarQ = 14;      // prepared query operands landed
constexpr int kBarM = 15;      // running max after tile i published and the one before it read (phase i)
constexpr int kSlotIssued = 16;  // int: producer's issued-tile mark (shares the slot area)
static_assert(kSlotIssued * 8 + 8 <= 192, "mbarrier area holds 24 slots");

constexpr float kLog2e = 1.4426950408889634f;
// 0x4B400000 read as fp32 is 1.5 * 2^23 = 12582912: an int32 accumulator started at this
// bias and moved by |x| < 2^22 reads as the exact float 12582912 + x
constexpr int kAccBias = 0x4B400000;
constexpr float kAccBiasF = 12582912.0f;

struct TensorMaps {
  CUtensorMap codes;  // cold codes  [tokens][2 x 128 B], box [2 blocks][128 rows][128 B]
  CUtensorMap crope;  // cold rope   [tokens][128 B], box [128 B][128 rows]
  CUtensorMap hlat;   // hot latent  [tokens][8 x 128 B], box [8 blocks][32 rows][128 B]
  CUtensorMap hrope;  // hot rope    [tokens][128 B], box [128 B][32 rows]
  CUtensorMap nlat;   // new latent  [total_q][8 x 128 B], box [8 blocks][32 rows][128 B]
  CUtensorMap nrope;  // new rope    [total_q][128 B], box [128 B][32 rows]
};

// ---------------------------------------------------------------------------
// mbarrier / TMA helpers
// ---------------------------------------------------------------------------
ASTERQ_DEVICE void tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// a [blocks][rows][128 B] box of a map whose third dimension steps through the 128-byte
// blocks of each row: one instruction for a tile's whole rows
ASTERQ_DEVICE void tma_3d(uint32_t dst, const CUtensorMap* map, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          dst),
      "l"(map), "r"(0), "r"(y), "r"(0), "r"(bar)
      : "memory");
}
// byte offset of (row, 16-byte chunk) in a [rows][128 B] region written with the
// 128-byte TMA swizzle: chunk index XOR (row mod 8)
ASTERQ_DEVICE int swz(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

struct Tile {
  int kind, page, off, n;
};

ASTERQ_DEVICE int4 fetch_tile(const asterq_decode_params& p, int idx) {
  return *reinterpret_cast<const int4*>(p.tiles + 4 * (int64_t)idx);
}

// Descriptor checks, applied when the tile is used: the main loops fetch the raw
// entry two tiles ahead and check it one tile ahead, so no warp waits on the load.
ASTERQ_DEVICE Tile check_tile(const asterq_decode_params& p, int4 t) {
  Tile tile{t.x, t.y, t.z, t.w};
  // a malformed entry reads nothing instead of faulting
  bool ok = tile.n > 0 && tile.off >= 0;
  if (tile.kind == ASTERQ_TILE_COLD) {
    ok = ok && tile.page >= 0 && tile.page < p.n_cold_pages &&
         tile.n <= (p.cold_scheme >= ASTERQ_SCHEME_INT8 ? kColdTile8 : kColdTile) && tile.off + tile.n <= p.page_tokens;
  } else if (tile.kind == ASTERQ_TILE_HOT) {
    ok = ok && tile.page >= 0 && tile.page < p.n_hot_pages && tile.n <= kHotTile && tile.off + tile.n <= p.page_tokens;
  } else if (tile.kind == ASTERQ_TILE_NEW) {
    ok = ok && tile.page >= 0 && tile.n <= kHotTile && (int64_t)tile.page + tile.off + tile.n <= p.total_q;
  } else {
    ok = false;
  }
  if (!ok) tile.n = 0;
  return tile;
}

ASTERQ_DEVICE Tile load_tile(const asterq_decode_params& p, int idx) { return check_tile(p, fetch_tile(p, idx)); }

// bound of every pipeline wait (asterq_decode_params.wait_limit_cycles; 0: the default)
ASTERQ_DEVICE long long wait_limit(const asterq_decode_params& p) {
  return (p.wait_limit_cycles > 0) ? p.wait_limit_cycles : kDefaultWaitLimit;
}

// Normalized FWHT of rows [r0, r0 + nrows) of a [16][512] fp32 buffer, one warp:
// lane l holds elements 16l..16l+15; stages h < 16 are lane-local, h >= 16 pair
// lane l with l ^ (h / 16).  Not on the bit-exact path.
ASTERQ_DEVICE void warp_fwht_rows(float* buf, int r0, int nrows, int lane) {
  for (int r = r0; r < r0 + nrows; ++r) {
    float v[16];
    float4* src = reinterpret_cast<float4*>(buf + r * kL + 16 * lane);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 x = src[k];
      v[4 * k] = x.x;
      v[4 * k + 1] = x.y;
      v[4 * k + 2] = x.z;
      v[4 * k + 3] = x.w;
    }
#pragma unroll
    for (int h = 1; h < 16; h <<= 1)
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (!(j & h)) {
          const float a = v[j], b = v[j + h];
          v[j] = a + b;
          v[j + h] = a - b;
        }
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
      const bool upper = (lane & m) != 0;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float o = __shfl_xor_sync(0xffffffffu, v[j], m);
        v[j] = upper ? (o - v[j]) : (v[j] + o);
      }
    }
    const float inv = 0.04419417382415922f;  // 1/sqrt(512)
#pragma unroll
    for (int k = 0; k < 4; ++k)
      src[k] = make_float4(v[4 * k] * inv, v[4 * k + 1] * inv, v[4 * k + 2] * inv, v[4 * k + 3] * inv);
  }
}

// Tile row (token) held at m-tile row r (0..15) of score-warp m-tile m.  Rows are
// permuted so that the 8-byte code loads of one instruction fall in distinct
// banks under the 128-byte swizzle: lanes gid 0..3 read rows 0,2,4,6 and gid 4..7
// read rows 1,3,5,7 of each 8-row group.
ASTERQ_DEVICE int qk_token(int warp, int m, int r) {
  const int g = r & 7;
  return 32 * warp + 16 * m + (((g & 3) << 1) | (g >> 2)) + (r & 8);
}

// ---------------------------------------------------------------------------
// Query preparation: one CTA per 16-row block (unit) writes the block's query
// operands to the workspace, in the layout of their shared-memory regions, so
// that every work item of the block starts with a 35 KB bulk copy instead of
// rotating and re-encoding the query itself.
//   qi      [16 k-steps][2 row tiles][32 lanes] uint4: rotated query as a per-row
//           16-bit fixed-point number split in two int8 limbs (cold QK B operand)
//   qh      [8 groups][4 k-steps][2][32] uint2: bf16 query x 2^e (hot QK B operand)
//   qr      [4][2][32] uint2: bf16 RoPE query x 2^e
//   scalars 2^e, 2^-e * scale, fixed-point scale, the two score multipliers
// ---------------------------------------------------------------------------
constexpr int kPrepThreads = 512;
constexpr int kPrepRowsPerWarp = kRows / (kPrepThreads / 32);  // one query row per warp
constexpr int kPrepSmem = 16 * kL * 4 + 16 * kL * 2 + 16 * kRope * 2 + 4 * kQScalars + 4 * (16 * kRope + 16);

__global__ void __launch_bounds__(kPrepThreads) qprep_kernel(const __grid_constant__ asterq_decode_params p) {
  extern __shared__ __align__(16) uint8_t prep_smem[];
  float* scratch = reinterpret_cast<float*>(prep_smem);                            // [16][512] fp32
  uint16_t* qraw = reinterpret_cast<uint16_t*>(prep_smem + 16 * kL * 4);           // [16][512] bf16
  uint16_t* rraw = reinterpret_cast<uint16_t*>(prep_smem + 16 * kL * 6);           // [16][64] bf16
  float* sc = reinterpret_cast<float*>(prep_smem + 16 * kL * 6 + 16 * kRope * 2);  // kQScalars, from kMQscale
  float* rscr = sc + kQScalars;  // quantized RoPE: [16][64] fp32 rotated RoPE query, then [16] fixed-point scales
  const bool rope_q = p.rope_scheme == ASTERQ_ROPE_QUANTIZED;
  const bool b8 = p.cold_scheme == ASTERQ_SCHEME_INT8;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int unit = blockIdx.x;
  // the decode grid may launch now; it waits for this grid's results before reading them
  asm volatile("griddepcontrol.launch_dependents;");
  if (p.plan_counts != nullptr && unit >= __ldg(p.plan_counts + 1)) return;  // beyond a device-built schedule
  const int64_t out_row0 = p.units[2 * unit];
  const int n_rows = min(max(p.units[2 * unit + 1], 0), kRows);
  uint8_t* dst = reinterpret_cast<uint8_t*>(p.workspace) + (int64_t)p.n_slots * kRecordBytes + (int64_t)unit * kQPrepBytes;
  // this call's fused-combine count of the unit starts at zero (the decode kernel runs after this kernel)
  if (tid == 0)
    reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(p.workspace) + counters_offset(p.n_slots, p.n_units))[unit] = 0;

  const uint16_t* ql = reinterpret_cast<const uint16_t*>(p.q_lat);
  const uint16_t* qrp = reinterpret_cast<const uint16_t*>(p.q_rope);
  for (int r = kPrepRowsPerWarp * warp; r < kPrepRowsPerWarp * (warp + 1); ++r) {
    float* d = scratch + r * kL + 16 * lane;
    uint4 a = make_uint4(0u, 0u, 0u, 0u), b = a, c = a;
    if (r < n_rows) {
      a = *reinterpret_cast<const uint4*>(ql + (out_row0 + r) * kL + 16 * lane);
      b = *reinterpret_cast<const uint4*>(ql + (out_row0 + r) * kL + 16 * lane + 8);
      if (lane < 8) c = *reinterpret_cast<const uint4*>(qrp + (out_row0 + r) * kRope + 8 * lane);
    }
    *reinterpret_cast<uint4*>(qraw + r * kL + 16 * lane) = a;
    *reinterpret_cast<uint4*>(qraw + r * kL + 16 * lane + 8) = b;
    if (lane < 8) *reinterpret_cast<uint4*>(rraw + r * kRope + 8 * lane) = c;
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      d[2 * k] = bf16lo_to_f32(w[k]);
      d[2 * k + 1] = bf16hi_to_f32(w[k]);
    }
  }
  __syncwarp();
  // hadamard_int4 scores the codes in the rotated basis (H q); plain int4 in the natural one
  if (p.cold_scheme == ASTERQ_SCHEME_HADAMARD_INT4) warp_fwht_rows(scratch, kPrepRowsPerWarp * warp, kPrepRowsPerWarp, lane);
  __syncwarp();
  for (int r = kPrepRowsPerWarp * warp; r < kPrepRowsPerWarp * (warp + 1); ++r) {
    float mx = 0.0f;
#pragma unroll
    for (int k = 0; k < 16; ++k) mx = fmaxf(mx, fabsf(scratch[r * kL + 16 * lane + k]));
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) {
      int e = 0;
      if (mx > 0.0f) {
        int ex;
        frexpf(mx, &ex);
        e = min(max(14 - ex, -100), 100);
      }
      const float qs = (mx > 0.0f) ? 32511.0f / mx : 1.0f;
      // INT4 codes enter the int8 MMAs as 16 x code (the nibble in the high half of the byte)
      const float cm = b8 ? 1.0f : 16.0f;
      sc[r] = ldexpf(1.0f, e);
      sc[kMQinv - kMQscale + r] = ldexpf(1.0f, -e) * p.softmax_scale;
      sc[kMQint - kMQscale + r] = qs;
      sc[kMQinvI - kMQscale + r] = p.softmax_scale / (cm * qs);
      sc[kMRopeR - kMQscale + r] = ldexpf(1.0f, -e) * (cm * qs);
    }
    if (rope_q) {
      // Quantized cold RoPE keys are scored like a ninth scale group: the RoPE query in the
      // codes' basis (normalized 64-point Hadamard for hadamard_int4: butterflies (a + b, a - b)
      // at distances 1, 2, .., 32, then / 8), with its own fixed-point scale; lane l holds
      // dims 2l and 2l + 1.
      const uint32_t w = *reinterpret_cast<const uint32_t*>(rraw + r * kRope + 2 * lane);
      float x0 = bf16lo_to_f32(w), x1 = bf16hi_to_f32(w);
      if (p.cold_scheme == ASTERQ_SCHEME_HADAMARD_INT4) {
        const float a = x0, b = x1;
        x0 = a + b;
        x1 = a - b;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
          const float o0 = __shfl_xor_sync(0xffffffffu, x0, d), o1 = __shfl_xor_sync(0xffffffffu, x1, d);
          const bool upper = (lane & d) != 0;
          x0 = upper ? o0 - x0 : x0 + o0;
          x1 = upper ? o1 - x1 : x1 + o1;
        }
        x0 *= 0.125f;
        x1 *= 0.125f;
      }
      rscr[r * kRope + 2 * lane] = x0;
      rscr[r * kRope + 2 * lane + 1] = x1;
      float rmx = fmaxf(fabsf(x0), fabsf(x1));
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) rmx = fmaxf(rmx, __shfl_xor_sync(0xffffffffu, rmx, off));
      if (lane == 0) {
        if (p.cold_scheme == ASTERQ_SCHEME_FLOAT8) {
          // float8: the RoPE query in fp16 times its own power of two (largest value below 2^14)
          int ex = 0;
          if (rmx > 0.0f) frexpf(rmx, &ex);
          const float s2r = ldexpf(1.0f, rmx > 0.0f ? min(max(14 - ex, -100), 100) : 0);
          rscr[16 * kRope + r] = s2r;
          sc[kMRopeR - kMQscale + r] = sc[r] / s2r;
        } else {
          const float qr_s = (rmx > 0.0f) ? 32511.0f / rmx : 1.0f;
          rscr[16 * kRope + r] = qr_s;
          sc[kMRopeR - kMQscale + r] = sc[kMQint - kMQscale + r] / qr_s;
        }
      }
    }
  }
  __syncthreads();
  // cold QK B fragments: k-step ks = 2 * group + j; lane (gid, tq) holds query row 8nt + gid at
  // k = 4tq + i (b0) and 16 + 4tq + i (b1), which the INT4 code expansion maps to dims 8W + 2i
  // and 8W + 2i + 1 of code word W = 8 * group + 2tq + j, and int8 codes to dims
  // 64 * group + 16tq + 8j + i and + 4 + i.  Two int8 limbs: q = 256 hi + lo.
  uint4* qi = reinterpret_cast<uint4*>(dst);
  if (p.cold_scheme == ASTERQ_SCHEME_FLOAT8) {
    // float8 codes are scored with fp16 MMAs: the same region holds the query in fp16 (times 2^e,
    // exact for a bf16 query), [group g][k-step ks][nt][lane] uint2, lane (gid, tq) holding row
    // 8nt + gid at dims 64g + 16tq + 4ks + {0, 1} (b0) and + {2, 3} (b1)
    uint2* qf = reinterpret_cast<uint2*>(dst);
    for (int e = tid; e < 8 * 4 * 2 * 32; e += kPrepThreads) {
      const int ln = e & 31, nt = (e >> 5) & 1, ks = (e >> 6) & 3, g = e >> 8;
      const int row = 8 * nt + (ln >> 2);
      const int d0 = 64 * g + 16 * (ln & 3) + 4 * ks;
      const float s2 = sc[row];
      const float2 f0 = unpack_bf162(*reinterpret_cast<const uint32_t*>(qraw + row * kL + d0));
      const float2 f1 = unpack_bf162(*reinterpret_cast<const uint32_t*>(qraw + row * kL + d0 + 2));
      qf[e] = make_uint2(pack_half2(f0.x * s2, f0.y * s2), pack_half2(f1.x * s2, f1.y * s2));
    }
  }
  for (int e = tid; e < 16 * 2 * 32 && p.cold_scheme != ASTERQ_SCHEME_FLOAT8; e += kPrepThreads) {
    const int ln = e & 31, nt = (e >> 5) & 1, ks = e >> 6;
    const int row = 8 * nt + (ln >> 2), W = 8 * (ks >> 1) + 2 * (ln & 3) + (ks & 1);
    const int d8 = 64 * (ks >> 1) + 16 * (ln & 3) + 8 * (ks & 1);
    const float qs = sc[kMQint - kMQscale + row];
    uint32_t hb[2] = {0u, 0u}, lb[2] = {0u, 0u};
#pragma unroll
    for (int half = 0; half < 2; ++half)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int dim = b8 ? d8 + 4 * half + i : 8 * W + 2 * i + half;
        const int qv = min(max(__float2int_rn(scratch[row * kL + dim] * qs), -32511), 32511);
        const int q1 = (qv + 128) >> 8;  // floor((q + 128) / 256): q1 in [-127, 127], q - 256 q1 in [-128, 127]
        const int q2 = qv - 256 * q1;
        hb[half] |= (uint32_t)(q1 & 0xff) << (8 * i);
        lb[half] |= (uint32_t)(q2 & 0xff) << (8 * i);
      }
    qi[e] = make_uint4(hb[0], hb[1], lb[0], lb[1]);
  }
  // hot-tile and RoPE bf16 fragments, in the order each consumer lane loads them
  uint2* qh = reinterpret_cast<uint2*>(dst + 16384);
  for (int e = tid; e < 8 * 4 * 2 * 32; e += kPrepThreads) {
    const int ln = e & 31, nt = (e >> 5) & 1, ks = (e >> 6) & 3, g = e >> 8;
    const int row = 8 * nt + (ln >> 2);
    const int e0 = 64 * g + 16 * ks + 2 * (ln & 3);
    const uint32_t w0 = *reinterpret_cast<const uint32_t*>(qraw + row * kL + e0);
    const uint32_t w1 = *reinterpret_cast<const uint32_t*>(qraw + row * kL + e0 + 8);
    const float s2 = sc[row];
    const float2 f0 = unpack_bf162(w0), f1 = unpack_bf162(w1);
    qh[e] = make_uint2(pack_bf162(f0.x * s2, f0.y * s2), pack_bf162(f1.x * s2, f1.y * s2));
  }
  uint2* qr = reinterpret_cast<uint2*>(dst + 32768);
  for (int e = tid; e < 4 * 2 * 32; e += kPrepThreads) {
    const int ln = e & 31, nt = (e >> 5) & 1, ks = e >> 6;
    const int row = 8 * nt + (ln >> 2);
    const int e0 = 16 * ks + 2 * (ln & 3);
    const uint32_t w0 = *reinterpret_cast<const uint32_t*>(rraw + row * kRope + e0);
    const uint32_t w1 = *reinterpret_cast<const uint32_t*>(rraw + row * kRope + e0 + 8);
    const float s2 = sc[row];
    const float2 f0 = unpack_bf162(w0), f1 = unpack_bf162(w1);
    qr[e] = make_uint2(pack_bf162(f0.x * s2, f0.y * s2), pack_bf162(f1.x * s2, f1.y * s2));
  }
  float* scalars = reinterpret_cast<float*>(dst + 34816);
  for (int e = tid; e < kQScalars; e += kPrepThreads) scalars[e] = sc[e];
  if (rope_q && p.cold_scheme == ASTERQ_SCHEME_FLOAT8) {
    // float8 RoPE codes: fp16 fragments [k-step ks][nt][lane] uint2, lane (gid, tq) holding row
    // 8nt + gid at RoPE dims 16tq + 4ks + {0, 1} (b0) and + {2, 3} (b1), times its power of two
    uint2* qfr = reinterpret_cast<uint2*>(dst + kQPrepRopeInt);
    for (int e = tid; e < 4 * 2 * 32; e += kPrepThreads) {
      const int ln = e & 31, nt = (e >> 5) & 1, ks = e >> 6;
      const int row = 8 * nt + (ln >> 2), d0 = 16 * (ln & 3) + 4 * ks;
      const float s2r = rscr[16 * kRope + row];
      const float* x = rscr + row * kRope + d0;
      qfr[e] = make_uint2(pack_half2(x[0] * s2r, x[1] * s2r), pack_half2(x[2] * s2r, x[3] * s2r));
    }
  } else if (rope_q) {
    // quantized RoPE limb fragments: k-step j, lane (gid, tq) holds query row 8nt + gid at the
    // dims of code word W = 2tq + j of the 32-byte INT4 RoPE code row (same expansion as the
    // latent), or for int8 RoPE codes at dims 16tq + 8j + i and + 4 + i
    uint4* qri = reinterpret_cast<uint4*>(dst + kQPrepRopeInt);
    for (int e = tid; e < 2 * 2 * 32; e += kPrepThreads) {
      const int ln = e & 31, nt = (e >> 5) & 1, j = e >> 6;
      const int row = 8 * nt + (ln >> 2), W = 2 * (ln & 3) + j;
      const float qs = rscr[16 * kRope + row];
      uint32_t hb[2] = {0u, 0u}, lb[2] = {0u, 0u};
#pragma unroll
      for (int half = 0; half < 2; ++half)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int rd = b8 ? 16 * (ln & 3) + 8 * j + 4 * half + i : 8 * W + 2 * i + half;
          const int qv = min(max(__float2int_rn(rscr[row * kRope + rd] * qs), -32511), 32511);
          const int q1 = (qv + 128) >> 8;
          const int q2 = qv - 256 * q1;
          hb[half] |= (uint32_t)(q1 & 0xff) << (8 * i);
          lb[half] |= (uint32_t)(q2 & 0xff) << (8 * i);
        }
      qri[e] = make_uint4(hb[0], hb[1], lb[0], lb[1]);
    }
  }
}

// Kernel instantiations (each mode's code and register allocation carry only its own path):
//  kModeInt4: INT4 codes (hadamard_int4 or int4) with bf16 RoPE keys;
//  kModeInt4RopeQ: INT4 codes with quantized RoPE keys (ASTERQ_ROPE_QUANTIZED);
//  kModeInt8: int8 codes (kv.py scheme "int8": one signed byte a dim, fp16 scale per group of 64),
//    bf16 RoPE keys, in 64-token cold tiles (512 code bytes a token: a tile holds as many code
//    bytes as a 128-token INT4 tile, so every warp's share of a stage is unchanged).
//  kModeF8: float8 e4m3 codes (kv.py scheme "float8": one byte a dim, no scales), bf16 RoPE keys,
//    64-token cold tiles like int8.
//  kModeInt8RopeQ / kModeF8RopeQ: the same with quantized RoPE keys (64 bytes a token: int8 codes
//    with one fp16 scale, or e4m3 bytes).
constexpr int kModeInt4 = 0, kModeInt4RopeQ = 1, kModeInt8 = 2, kModeF8 = 3, kModeInt8RopeQ = 4, kModeF8RopeQ = 5;
template <int kMode>
__global__ void __launch_bounds__(kThreads, 1)
    decode_kernel(const __grid_constant__ asterq_decode_params p, const __grid_constant__ TensorMaps maps) {
  constexpr bool kRopeQ = kMode == kModeInt4RopeQ || kMode == kModeInt8RopeQ || kMode == kModeF8RopeQ;
  constexpr bool kB8 = kMode == kModeInt8 || kMode == kModeInt8RopeQ;
  constexpr bool kF8 = kMode == kModeF8 || kMode == kModeF8RopeQ;
  constexpr bool kBytes = kB8 || kF8;                   // one code byte a dim, 64-token cold tiles
  constexpr int kCT = kBytes ? kColdTile8 : kColdTile;  // tokens of a cold tile
  constexpr int kCM = kCT / 64;                      // 16-token m-tiles of a cold tile per score warp
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base, derived by indexing the __shared__ array so that the
  // compiler keeps every access through `smem` in the shared state space
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  float* misc = reinterpret_cast<float*>(smem + kOffMisc);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + kBarAbort);
  auto bar = [&](int i) { return smem_u32(bars + i); };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, tq = lane & 3;
  const int H = p.n_heads;
  // This CTA's work items: one (item blockIdx.x) without a worker table, else the
  // contiguous range workers[blockIdx.x] .. workers[blockIdx.x + 1], run one after another.
  int it_begin = blockIdx.x, it_end = blockIdx.x + 1;
  if (p.workers != nullptr) {
    it_begin = max(p.workers[blockIdx.x], 0);
    it_end = min(p.workers[blockIdx.x + 1], p.n_items);
  }
  // fields of the current item (begin_item)
  const int* itm = p.items;
  int rb = 0, tile_begin = 0, slot = -2, n_rows = 0, n_t = 0;
  int64_t out_row0 = 0;
  // producer lane: one past the last tile of the current item it has requested (shared memory)
  volatile int* issued_hi = reinterpret_cast<volatile int*>(bars + kSlotIssued);
  auto begin_item = [&](int it) {
    itm = p.items + 8 * (int64_t)it;
    rb = itm[1];
    tile_begin = max(itm[2], 0);
    const int tile_end = max(min(itm[3], p.n_tiles), tile_begin);
    slot = (itm[4] < p.n_slots) ? itm[4] : -2;  // -2: out-of-range slot, write nothing
    out_row0 = itm[5];
    n_rows = min(itm[6], kRows);
    n_t = tile_end - tile_begin;
  };

  // every item starts from freshly initialized barriers (the previous item's are
  // quiescent: each of its copies was waited for before the CTA-wide barrier)
  auto init_barriers = [&](bool again) {
    if (again) {
#pragma unroll 1
      for (int k = 0; k <= kBarM; ++k)
        if (k != kBarAbort) mbar_inval(bar(k));
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kBarEmpty + s), 32 * (kTeamWarps + kValueWarps));
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(kBarPFull + b), 32 * kTeamWarps);
      mbar_init(bar(kBarPEmpty + b), 32 * kValueWarps);
    }
    for (int f = 0; f < kFullBars; ++f) mbar_init(bar(kBarFull + f), 1);
    mbar_init(bar(kBarQ), 1);
    mbar_init(bar(kBarM), 32 * kTeamWarps);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  };
  if (tid == 0) init_barriers(false);
  __syncthreads();
  // between two items: the previous epilogue is done everywhere, then thread 0 resets the barriers
  auto next_item_sync = [&]() {
    named_sync(0, kThreads);
    if (tid == 0) init_barriers(true);
    named_sync(0, kThreads);
  };

  // ---------------- producer: issue one tile into its stage ----------------
  auto issue_tile = [&](int j, const Tile t) {
    const int s = j % kStages;
    const uint32_t full = bar(kBarFull + j % kFullBars);
    const uint32_t st = sbase + s * kStageBytes;
    if (t.kind == ASTERQ_TILE_HOLD) return;  // test hook: never arrives (the waits for it time out)
    *issued_hi = j + 1;
    if (t.n == 0) {
      mbar_arrive(full);
      return;
    }
    if (t.kind == ASTERQ_TILE_COLD) {
      const int y = t.page * p.page_tokens + t.off;
      if constexpr (kRopeQ) {
        // RoPE codes (32 B a token for INT4, 64 B for int8 / float8) and, but for float8, their
        // scales (2 B a token, copied from the 8-token boundary at or below y to the one at or
        // above y + n: both within the page, whose first token index is a multiple of 16)
        constexpr int kRB = kBytes ? 64 : 32;
        const int y8 = y & ~7, n8 = ((y + t.n + 7) & ~7) - y8;
        mbar_expect_tx(full, (kBytes ? 4 * kCodeBlock8 : 2 * 16384) + (kF8 ? 0 : 16 * t.n + 2 * n8) + kRB * t.n);
        tma_3d(st + kCodesLo, &maps.codes, y, full);
        bulk_1d(st + kCRope, reinterpret_cast<const uint8_t*>(p.cold_rope) + (int64_t)y * kRB, kRB * t.n, full);
        if constexpr (!kF8)
          bulk_1d(st + kCRopeScale, reinterpret_cast<const uint8_t*>(p.cold_rope_scales) + (int64_t)y8 * 2, 2 * n8, full);
      } else if constexpr (kBytes) {
        mbar_expect_tx(full, 4 * kCodeBlock8 + kColdTile8 * 128 + (kF8 ? 0 : 16 * t.n));
        tma_3d(st + kCodesLo, &maps.codes, y, full);  // four blocks of [64 rows][128 B]
        tma_2d(st + kCRope, &maps.crope, 0, y, full);
      } else {
        mbar_expect_tx(full, 3 * 16384 + 16 * t.n);
        tma_3d(st + kCodesLo, &maps.codes, y, full);  // both halves: kCodesHi = kCodesLo + 128 rows x 128 B
        tma_2d(st + kCRope, &maps.crope, 0, y, full);
      }
      if constexpr (!kF8)
        bulk_1d(st + kScales, reinterpret_cast<const uint8_t*>(p.cold_scales) + (int64_t)y * 16, 16 * t.n, full);
    } else {
      const bool hot = t.kind == ASTERQ_TILE_HOT;
      const int y = hot ? t.page * p.page_tokens + t.off : t.page + t.off;
      const CUtensorMap* lat = hot ? &maps.hlat : &maps.nlat;
      mbar_expect_tx(full, 9 * 4096);
      tma_3d(st, lat, y, full);  // block g lands at g * kHotBlock
      tma_2d(st + kHRope, hot ? &maps.hrope : &maps.nrope, 0, y, full);
    }
  };
  auto issue = [&](int j) { issue_tile(j, load_tile(p, tile_begin + j)); };
  // ---------------- prologue (producer lane): first tiles and the prepared query ----------------
  // (qprep_kernel wrote the query operands to the workspace: int8 limb fragments, hot and
  // RoPE bf16 fragments, per-row scalars, laid out like their shared-memory regions)
  // (the query block first: it comes from L2 and gates every tile, the tiles come from HBM;
  // the CTA's first item has its tiles in flight already, see below)
  auto prologue = [&](bool tiles_issued) {
    if (!tiles_issued) *issued_hi = 0;
    const uint8_t* src = reinterpret_cast<const uint8_t*>(p.workspace) + (int64_t)p.n_slots * kRecordBytes +
                         (int64_t)max(itm[0], 0) * kQPrepBytes;
    const uint32_t qb = bar(kBarQ);
    constexpr bool rope_q = kRopeQ;
    mbar_expect_tx(qb, kQPrepCopyBytes + (rope_q ? 2048u : 0u));
    bulk_1d(sbase + kOffQi, src, 16384, qb);
    bulk_1d(sbase + kOffQh, src + 16384, 16384, qb);
    bulk_1d(sbase + kOffQr, src + 32768, 2048, qb);
    bulk_1d(sbase + kOffMisc + 4 * kMQscale, src + 34816, 4 * kQScalars, qb);
    if (rope_q) bulk_1d(sbase + kOffQri, src + kQPrepRopeInt, 2048, qb);
    if (!tiles_issued)
      for (int j = 0; j < min(n_t, kStages); ++j) issue(j);
  };
  // This grid may start while qprep_kernel still runs (programmatic dependent launch): the
  // first item's tiles read only the cache, so they are requested before every thread
  // waits for qprep_kernel's results (the query blocks and the unit counters).
  if (warp == kProducerWarp && lane == 0 && it_begin < it_end) {
    *issued_hi = 0;
    begin_item(it_begin);
    for (int j = 0; j < min(n_t, kStages); ++j) issue(j);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---------------- epilogue: normalize or write the partial record ----------------
  // (after a CTA-wide barrier; returns true when a wait of this item timed out: the CTA
  // then records the failure and stops)
  auto epilogue = [&]() -> bool {
    const float* O = reinterpret_cast<const float*>(smem + kOffQi);
    const float* lw = misc + kMLw;
    const float* mrow = misc + kMWmax;
    if (slot == -1) {
      for (int e = tid; e < kRows * kL / 4; e += kThreads) {
        const int r = e >> 7, c4 = e & 127;
        if (r >= n_rows) continue;
        float l = 0.0f;
#pragma unroll
        for (int w2 = 0; w2 < kScoreWarps; ++w2) l += lw[16 * w2 + r];
        const float inv = 1.0f / fmaxf(l, 1e-20f);
        const float4 v = *reinterpret_cast<const float4*>(O + r * kL + 4 * c4);
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
      for (int e = tid; e < kRows * kL / 4; e += kThreads) {
        const int r = e >> 7, c4 = e & 127;
        *reinterpret_cast<float4*>(wo + ((int64_t)slot * kRows + r) * kL + 4 * c4) =
            *reinterpret_cast<const float4*>(O + r * kL + 4 * c4);
      }
      if (tid < kRows) {
        wm[(int64_t)slot * kRows + tid] = mrow[tid];
        float l = 0.0f;
#pragma unroll
        for (int w2 = 0; w2 < kScoreWarps; ++w2) l += lw[16 * w2 + tid];
        wl[(int64_t)slot * kRows + tid] = l;
      }
      // Fused combine job of this unit: every CTA that writes one of its partial records
      // counts it; the one that writes the last merges them all (latent_attention.py:212-220
      // applied across splits, as combine_kernel does), so no separate launch is needed.
      const int unit = itm[0];
      const int job = (p.unit_jobs != nullptr && unit >= 0 && unit < p.n_units) ? p.unit_jobs[unit] : -1;
      const int first_fused = (p.plan_counts != nullptr) ? __ldg(p.plan_counts + 6) : p.n_combine;
      if (job >= first_fused && job < p.n_combine_total) {
        const int4 jb = *reinterpret_cast<const int4*>(p.combine + 4 * (int64_t)job);
        const int s0 = max(jb.x, 0), s1 = min(jb.y, p.n_slots), rows = min(jb.w, kRows);
        __threadfence();  // this CTA's record is visible device-wide before the count moves
        named_sync(0, kThreads);
        volatile int* last = reinterpret_cast<volatile int*>(misc + kMAlpha);
        if (tid == 0) {
          int* ctr = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(p.workspace) + counters_offset(p.n_slots, p.n_units));
          *last = atomicAdd(ctr + unit, 1) == s1 - s0 - 1;
        }
        named_sync(0, kThreads);
        if (*last) {
          __threadfence();
          const int n_parts = s1 - s0;
          if (tid < kRows) {
            float mmax = -INFINITY;
            for (int q = s0; q < s1; ++q) mmax = fmaxf(mmax, __ldcg(wm + (int64_t)q * kRows + tid));
            const float msub = (mmax == -INFINITY) ? 0.0f : mmax;
            float l = 0.0f;
            for (int q = s0; q < s1; ++q)
              l += exp2f((__ldcg(wm + (int64_t)q * kRows + tid) - msub) * kLog2e) * __ldcg(wl + (int64_t)q * kRows + tid);
            misc[kMComb + tid] = msub;
            misc[kMComb + kRows + tid] = 1.0f / fmaxf(l, 1e-20f);
          }
          // this thread's four outputs (rows r0 + 4j, 4 dims at c4), accumulated over the parts
          // eight at a time: weights w_q / l of the eight parts in shared memory, then the
          // eight records' loads issued together
          const int r0 = tid >> 7, c4 = tid & 127;
          float4 acc[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          float* wq = misc + kMComb + 2 * kRows;  // [8 parts][16 rows]
          for (int c = 0; c < n_parts; c += 8) {
            named_sync(0, kThreads);  // row scalars written / previous weights consumed
            if (tid < 8 * kRows) {
              const int q = c + (tid >> 4), r = tid & 15;
              wq[tid] = (q < n_parts) ? exp2f((__ldcg(wm + (int64_t)(s0 + q) * kRows + r) - misc[kMComb + r]) * kLog2e) *
                                            misc[kMComb + kRows + r]
                                      : 0.0f;
            }
            named_sync(0, kThreads);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              if (c + q >= n_parts) break;
              const float* rec = wo + (int64_t)(s0 + c + q) * kRows * kL;
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int r = r0 + 4 * j;
                const float w = wq[q * kRows + r];
                const float4 v = __ldcg(reinterpret_cast<const float4*>(rec + r * kL + 4 * c4));
                acc[j].x += w * v.x;
                acc[j].y += w * v.y;
                acc[j].z += w * v.z;
                acc[j].w += w * v.w;
              }
            }
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int r = r0 + 4 * j;
            if (r >= rows) continue;
            const int64_t off = ((int64_t)jb.z + r) * kL + 4 * c4;
            if (p.out_dtype == ASTERQ_DTYPE_F32) {
              *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + off) = acc[j];
            } else {
              *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.out) + off) =
                  make_uint2(pack_bf162(acc[j].x, acc[j].y), pack_bf162(acc[j].z, acc[j].w));
            }
          }
        }
      }
    }
    const bool stop = *abort_flag != 0;
    if (tid == 0 && stop && p.device_status) atomicExch(p.device_status, 1);
    return stop;
  };

  if (warp < kScoreWarps) {
    // =====================================================================
    // score warps
    // =====================================================================
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kBytes ? kScoreRegsB : kScoreRegs));
    // team `team` takes tiles team, team + 2, ...; tw is the warp's index in its team
    const int team = warp / kTeamWarps, tw = warp % kTeamWarps;
    // cold tile token of accumulator row r (0..15) of this warp's m-tile m: INT4 tiles give each
    // warp 32 tokens in a code-word-derived order, int8 tiles 16 tokens in order
    auto ctok = [&](int m, int r) { return kBytes ? 16 * tw + r : qk_token(tw, m, r); };
#pragma unroll 1
    for (int it = it_begin; it < it_end; ++it) {
      begin_item(it);
      if (it > it_begin) next_item_sync();
      mbar_wait(bar(kBarQ), 0, abort_flag, wait_limit(p));
      const uint2* qh = reinterpret_cast<const uint2*>(smem + kOffQh);
      const uint2* qr = reinterpret_cast<const uint2*>(smem + kOffQr);
      float qinv[2][2], qinvi[2][2], rratio[2][2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          qinv[nt][cc] = misc[kMQinv + 8 * nt + 2 * tq + cc];
          qinvi[nt][cc] = misc[kMQinvI + 8 * nt + 2 * tq + cc];
          rratio[nt][cc] = misc[kMRopeR + 8 * nt + 2 * tq + cc];
        }
      // Softmax state of rows 8nt + 2tq + cc, replicated across the 8 gid lanes.  The running
      // max is one chain over all tiles: the team of tile i reads the max after tile i - 1
      // from the other team (kBarM phase i - 1) and publishes its own (phase i), so one team's
      // QK of its next tile overlaps the other team's softmax.  Each team sums its own tiles'
      // p relative to the max after its latest tile (m_team); both sums are brought to the
      // final max at the end.
      float m_team[2][2], l_w[2][2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          m_team[nt][cc] = -INFINITY;
          l_w[nt][cc] = 0.0f;
        }

      Tile t_next = (team < n_t) ? load_tile(p, tile_begin + team) : Tile{ASTERQ_TILE_HOT, 0, 0, 0};
      int4 raw_next = (team + 2 < n_t) ? fetch_tile(p, tile_begin + team + 2) : make_int4(0, 0, 0, 0);
#pragma unroll 1
      for (int i = team; i < n_t; i += 2) {
        const int s = i % kStages, b = i & 1;
        const Tile t = t_next;
        // descriptors: this team's next tile checked (fetched a tile ago), the one after fetched
        if (i + 2 < n_t) t_next = check_tile(p, raw_next);
        if (i + 4 < n_t) raw_next = fetch_tile(p, tile_begin + i + 4);
        mbar_wait(bar(kBarFull + i % kFullBars), (i / kFullBars) & 1, abort_flag, wait_limit(p));
        const uint8_t* st = smem + s * kStageBytes;
        const uint32_t sst = sbase + s * kStageBytes;
        const bool cold = t.kind == ASTERQ_TILE_COLD;
        float S[2][2][4];
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int c = 0; c < 4; ++c) S[m][nt][c] = 0.0f;

        if (cold) {
          int tok[2][2];
#pragma unroll
          for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int h = 0; h < 2; ++h) tok[m][h] = ctok(m, gid + 8 * h);
          const __half* scl = reinterpret_cast<const __half*>(st + kScales);
          if constexpr (kRopeQ) {
            // quantized RoPE keys: scored as a ninth scale group in the group loop below
          } else {
            // RoPE channel first (bf16, exact products), moved into the integer-score units
#pragma unroll
            for (int m = 0; m < kCM; ++m) {
              const int row = ctok(m, (lane & 7) + 8 * ((lane >> 3) & 1));
#pragma unroll
              for (int ks = 0; ks < 4; ++ks) {
                uint32_t a[4];
                ldmatrix_x4(a, sst + kCRope + swz(row, 2 * ks + (lane >> 4)));
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                  const uint2 bq = qr[(ks * 2 + nt) * 32 + lane];
                  mma_bf16(S[m][nt], a, bq.x, bq.y);
                }
              }
            }
            if constexpr (!kF8) {  // float8 scores stay in the hot tiles' units (qinv)
#pragma unroll
              for (int m = 0; m < 2; ++m)
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                  for (int c = 0; c < 4; ++c) S[m][nt][c] *= rratio[nt][c & 1];
            }
          }
          if constexpr (kF8) {
            // float8 codes: fp16 MMAs (m16n8k16) of the exact fp16 values of the e4m3 bytes against
            // the query in fp16 (the bf16 query times 2^e, exact); no scales.  Lane tq's 16 bytes of
            // group g (dims 64g + 16tq .. + 15) of its two tokens; k-step ks takes dims
            // 16tq + 4ks + {0, 1} (a0 / b0) and + {2, 3} (a2 / b1)
            const uint2* qf = reinterpret_cast<const uint2*>(smem + kOffQi);
            if constexpr (kRopeQ) {
              // quantized RoPE keys (e4m3 bytes, 64 a token) first, against the RoPE query in fp16
              // with its own power-of-two scale, then brought to the latent query's scale
              const uint2* qfr = reinterpret_cast<const uint2*>(smem + kOffQri);
              const uint4 r0 = *reinterpret_cast<const uint4*>(st + kCRope + 64 * tok[0][0] + 16 * tq);
              const uint4 r1 = *reinterpret_cast<const uint4*>(st + kCRope + 64 * tok[0][1] + 16 * tq);
#pragma unroll
              for (int ks = 0; ks < 4; ++ks) {
                const uint32_t w0 = ks == 0 ? r0.x : ks == 1 ? r0.y : ks == 2 ? r0.z : r0.w;
                const uint32_t w1 = ks == 0 ? r1.x : ks == 1 ? r1.y : ks == 2 ? r1.z : r1.w;
                const uint32_t a[4] = {e4m3x2_to_f16x2(w0), e4m3x2_to_f16x2(w1), e4m3x2_to_f16x2(w0 >> 16),
                                       e4m3x2_to_f16x2(w1 >> 16)};
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                  const uint2 bq = qfr[(ks * 2 + nt) * 32 + lane];
                  mma_f16(S[0][nt], a, bq.x, bq.y);
                }
              }
#pragma unroll
              for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int c = 0; c < 4; ++c) S[0][nt][c] *= rratio[nt][c & 1];
            }
#pragma unroll 2
            for (int g = 0; g < 8; ++g) {
              uint4 v[2];
#pragma unroll
              for (int h = 0; h < 2; ++h)
                v[h] = *reinterpret_cast<const uint4*>(st + (g >> 1) * kCodeBlock8 + swz(tok[0][h], 4 * (g & 1) + tq));
#pragma unroll
              for (int ks = 0; ks < 4; ++ks) {
                const uint32_t w0 = ks == 0 ? v[0].x : ks == 1 ? v[0].y : ks == 2 ? v[0].z : v[0].w;
                const uint32_t w1 = ks == 0 ? v[1].x : ks == 1 ? v[1].y : ks == 2 ? v[1].z : v[1].w;
                const uint32_t a[4] = {e4m3x2_to_f16x2(w0), e4m3x2_to_f16x2(w1), e4m3x2_to_f16x2(w0 >> 16),
                                       e4m3x2_to_f16x2(w1 >> 16)};
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                  const uint2 bq = qf[((g * 4 + ks) * 2 + nt) * 32 + lane];
                  mma_f16(S[0][nt], a, bq.x, bq.y);
                }
              }
            }
          } else {
            const uint4* qi = reinterpret_cast<const uint4*>(smem + kOffQi);
            // Group g's integer dot products (two int8 limbs of the query, both k-steps):
            // loads, code expansion and 16 MMAs into acc.
            auto qk_issue = [&](int g, int (&acc)[2][2][2][4]) {
              if constexpr (kB8) {
                // int8 codes: lane tq's 16 bytes of group g (dims 64g + 16tq .. + 15) of each of its
                // two tokens; k-step j takes dims 16tq + 8j + {0..3} (b0) and + {4..7} (b1), the
                // order the query limbs were laid out in
                uint4 v[2];
  #pragma unroll
                for (int h = 0; h < 2; ++h)  // group 8: the token's 64-byte RoPE code row (quantized RoPE keys)
                  v[h] = *reinterpret_cast<const uint4*>(st + ((kRopeQ && g == 8) ? kCRope + 64 * tok[0][h] + 16 * tq
                                                                                  : (g >> 1) * kCodeBlock8 + swz(tok[0][h], 4 * (g & 1) + tq)));
  #pragma unroll
                for (int j = 0; j < 2; ++j) {
                  const uint4 bq[2] = {qi[((2 * g + j) * 2) * 32 + lane], qi[((2 * g + j) * 2 + 1) * 32 + lane]};
                  const uint32_t a[4] = {j ? v[0].z : v[0].x, j ? v[1].z : v[1].x, j ? v[0].w : v[0].y, j ? v[1].w : v[1].y};
  #pragma unroll
                  for (int nt = 0; nt < 2; ++nt) {
                    if (j == 0) {
                      mma_s8_from(acc[0][0][nt], a, bq[nt].x, bq[nt].y, kAccBias);
                      mma_s8_from(acc[1][0][nt], a, bq[nt].z, bq[nt].w, kAccBias);
                    } else {
                      mma_s8(acc[0][0][nt], a, bq[nt].x, bq[nt].y);
                      mma_s8(acc[1][0][nt], a, bq[nt].z, bq[nt].w);
                    }
                  }
                }
                return;
              }
              // code words 8g + 2tq (k-step 2g) and 8g + 2tq + 1 (k-step 2g + 1) of the four tokens;
              // group 8 (quantized RoPE keys): words 2tq and 2tq + 1 of the token's 32-byte RoPE code
              // row, whose query limbs follow those of group 7 (k-steps 16 and 17)
              const int region = (g < 4) ? kCodesLo : kCodesHi;
              const int chunk = 2 * (g & 3) + (tq >> 1);
              uint2 v[2][2];
  #pragma unroll
              for (int m = 0; m < 2; ++m)
  #pragma unroll
                for (int h = 0; h < 2; ++h) {
                  const int off = (kRopeQ && g == 8) ? kCRope + 32 * tok[m][h] + 8 * tq
                                                     : region + swz(tok[m][h], chunk) + 8 * (tq & 1);
                  v[m][h] = *reinterpret_cast<const uint2*>(st + off);
                }
  #pragma unroll
              for (int j = 0; j < 2; ++j) {
                const uint4 bq[2] = {qi[((2 * g + j) * 2) * 32 + lane], qi[((2 * g + j) * 2 + 1) * 32 + lane]};
  #pragma unroll
                for (int m = 0; m < 2; ++m) {
                  const uint32_t x0 = j ? v[m][0].y : v[m][0].x, x1 = j ? v[m][1].y : v[m][1].x;
                  const uint32_t a[4] = {s8_lo_nibbles(x0), s8_lo_nibbles(x1), s8_hi_nibbles(x0), s8_hi_nibbles(x1)};
  #pragma unroll
                  for (int nt = 0; nt < 2; ++nt) {
                    if (j == 0) {
                      mma_s8_from(acc[0][m][nt], a, bq[nt].x, bq[nt].y, kAccBias);
                      mma_s8_from(acc[1][m][nt], a, bq[nt].z, bq[nt].w, kAccBias);
                    } else {
                      mma_s8(acc[0][m][nt], a, bq[nt].x, bq[nt].y);
                      mma_s8(acc[1][m][nt], a, bq[nt].z, bq[nt].w);
                    }
                  }
                }
              }
            };
            // S += scale_g x (256 hi + lo + B), the biased accumulators read as exact floats
            // (packed f32x2 arithmetic: two accumulator elements per instruction; elements
            // c = 0,1 belong to token row gid, c = 2,3 to row gid + 8).  The hi limb's bias B is
            // subtracted exactly; the lo limb keeps its bias, so each token's S carries
            // B x (sum of its group scales), subtracted once after the last group (|S| stays
            // below ~2^27 x scale, so the extra rounding is ~2^-21 of the score).
            float ssum[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
            auto qk_finish = [&](int g, const int (&acc)[2][2][2][4]) {
              const float2 bias2 = make_float2(-kAccBiasF, -kAccBiasF), k256 = make_float2(256.0f, 256.0f);
  #pragma unroll
              for (int m = 0; m < kCM; ++m) {
                const float s0 = __half2float(scl[8 * tok[m][0] + g]);
                const float s1 = __half2float(scl[8 * tok[m][1] + g]);
                ssum[m][0] += s0;
                ssum[m][1] += s1;
  #pragma unroll
                for (int nt = 0; nt < 2; ++nt)
  #pragma unroll
                  for (int h = 0; h < 2; ++h) {
                    const float2 fh = add2(make_float2(__int_as_float(acc[0][m][nt][2 * h]), __int_as_float(acc[0][m][nt][2 * h + 1])), bias2);
                    const float2 fl = make_float2(__int_as_float(acc[1][m][nt][2 * h]), __int_as_float(acc[1][m][nt][2 * h + 1]));
                    const float sc = h ? s1 : s0;
                    const float2 r = fma2(fma2(fh, k256, fl), make_float2(sc, sc),
                                          make_float2(S[m][nt][2 * h], S[m][nt][2 * h + 1]));
                    S[m][nt][2 * h] = r.x;
                    S[m][nt][2 * h + 1] = r.y;
                  }
              }
            };
            // two groups in flight: group g + 1's MMAs run on the tensor pipe while
            // group g's accumulators are scaled into S
            int accA[2][2][2][4], accB[2][2][2][4];
            if constexpr (kRopeQ) {
              // group 8, the quantized RoPE keys, first: its MMAs overlap group 0's, then
              // S = (256 hi + lo) x token scale x (latent / RoPE fixed-point scales), both limbs'
              // biases subtracted exactly (packed f32x2: elements 2h, 2h + 1 are token tok[m][h]
              // against rows 8nt + 2tq + {0, 1})
              qk_issue(8, accB);
              qk_issue(0, accA);
              // (the scales were copied from the 8-token boundary below the tile's first token
              // page * page_tokens + off; page_tokens is a multiple of 16, so that is off & 7 tokens back)
              const __half* rsc = reinterpret_cast<const __half*>(st + kCRopeScale) + (t.off & 7);
              const float2 bias2 = make_float2(-kAccBiasF, -kAccBiasF), k256 = make_float2(256.0f, 256.0f);
  #pragma unroll
              for (int m = 0; m < kCM; ++m)
  #pragma unroll
                for (int h = 0; h < 2; ++h) {
                  const float rs = __half2float(rsc[tok[m][h]]);
  #pragma unroll
                  for (int nt = 0; nt < 2; ++nt) {
                    const float2 fh = add2(make_float2(__int_as_float(accB[0][m][nt][2 * h]), __int_as_float(accB[0][m][nt][2 * h + 1])), bias2);
                    const float2 fl = add2(make_float2(__int_as_float(accB[1][m][nt][2 * h]), __int_as_float(accB[1][m][nt][2 * h + 1])), bias2);
                    const float2 w = mul2(make_float2(rs, rs), make_float2(rratio[nt][0], rratio[nt][1]));
                    const float2 r = mul2(fma2(fh, k256, fl), w);
                    S[m][nt][2 * h] = r.x;
                    S[m][nt][2 * h + 1] = r.y;
                  }
                }
            } else {
              qk_issue(0, accA);
            }
  #pragma unroll 1
            for (int g = 0; g < 8; g += 2) {
              qk_issue(g + 1, accB);
              qk_finish(g, accA);
              if (g + 2 < 8) qk_issue(g + 2, accA);
              qk_finish(g + 1, accB);
            }
            // the lo limbs' bias: B x (sum of the token's group scales)
  #pragma unroll
            for (int m = 0; m < kCM; ++m)
  #pragma unroll
              for (int nt = 0; nt < 2; ++nt)
  #pragma unroll
                for (int h = 0; h < 2; ++h) {
                  const float corr = -kAccBiasF * ssum[m][h];
                  S[m][nt][2 * h] += corr;
                  S[m][nt][2 * h + 1] += corr;
                }
          }
        } else {
          if constexpr (kBytes) {
            // hot / new tile (32 tokens), byte-code modes: warp tw scores all 32 tokens (two full
            // m-tiles) over scale groups 2tw and 2tw + 1 and RoPE k-step tw; the four partial scores
            // meet in the stage's tail (a hot tile's bf16 data ends at kHotPartial) and warp tw sums
            // the rows of its own 8 tokens 8tw + gid, the layout the softmax below reads.  (The
            // INT4 modes keep the form below, which measured faster there.)
            float part[2][2][2][4];  // [group of the pair][m-tile][nt][c]
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2)
#pragma unroll
              for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                  for (int c = 0; c < 4; ++c) part[h2][mt][nt][c] = 0.0f;
            const int lrow = (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
#pragma unroll
              for (int h2 = 0; h2 < 2; ++h2) {
                const int g = 2 * tw + h2;
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                  uint32_t a[4];
                  ldmatrix_x4(a, sst + g * kHotBlock + swz(16 * mt + lrow, 2 * ks + (lane >> 4)));
#pragma unroll
                  for (int nt = 0; nt < 2; ++nt) {
                    const uint2 bq = qh[((g * 4 + ks) * 2 + nt) * 32 + lane];
                    mma_bf16(part[h2][mt][nt], a, bq.x, bq.y);
                  }
                }
              }
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
              uint32_t a[4];
              ldmatrix_x4(a, sst + kHRope + swz(16 * mt + lrow, 2 * tw + (lane >> 4)));
#pragma unroll
              for (int nt = 0; nt < 2; ++nt) {
                const uint2 bq = qr[(tw * 2 + nt) * 32 + lane];
                mma_bf16(part[1][mt][nt], a, bq.x, bq.y);
              }
            }
            // partial scores [warp][token][row] (row stride kPartStride floats) in the stage's tail
            float* xbuf = reinterpret_cast<float*>(smem + s * kStageBytes + kHotPartial);
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
              for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  const int token = 16 * mt + gid + 8 * h;
                  *reinterpret_cast<float2*>(xbuf + (tw * kHotTile + token) * kPartStride + 8 * nt + 2 * tq) =
                      make_float2(part[0][mt][nt][2 * h] + part[1][mt][nt][2 * h],
                                  part[0][mt][nt][2 * h + 1] + part[1][mt][nt][2 * h + 1]);
                }
            named_sync(1 + team, 32 * kTeamWarps);
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
              float2 sum = make_float2(0.0f, 0.0f);
#pragma unroll
              for (int w = 0; w < kTeamWarps; ++w) {
                const float2 v =
                    *reinterpret_cast<const float2*>(xbuf + (w * kHotTile + 8 * tw + gid) * kPartStride + 8 * nt + 2 * tq);
                sum.x += v.x;
                sum.y += v.y;
              }
              S[0][nt][0] = sum.x;
              S[0][nt][1] = sum.y;
            }
            // these generic-proxy writes precede the next TMA write of this stage (after its release)
            fence_async_shared();
          } else {
            // hot / new tile: this warp's 8 tokens fill m-tile rows 0-7 (rows 8-15 repeat them);
            // S[1] is a second partial accumulator (odd groups) folded in below
            const int row = 8 * tw + (lane & 7);
  #pragma unroll 1
            for (int g = 0; g < 8; g += 2) {
  #pragma unroll
              for (int ks = 0; ks < 4; ++ks) {
                uint32_t a[2][4];
                ldmatrix_x4(a[0], sst + g * kHotBlock + swz(row, 2 * ks + (lane >> 4)));
                ldmatrix_x4(a[1], sst + (g + 1) * kHotBlock + swz(row, 2 * ks + (lane >> 4)));
  #pragma unroll
                for (int h2 = 0; h2 < 2; ++h2)
  #pragma unroll
                  for (int nt = 0; nt < 2; ++nt) {
                    const uint2 bq = qh[(((g + h2) * 4 + ks) * 2 + nt) * 32 + lane];
                    mma_bf16(S[h2][nt], a[h2], bq.x, bq.y);
                  }
              }
            }
  #pragma unroll
            for (int nt = 0; nt < 2; ++nt)
  #pragma unroll
              for (int c = 0; c < 4; ++c) {
                S[0][nt][c] += S[1][nt][c];
                S[1][nt][c] = 0.0f;
              }
  #pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              uint32_t a[4];
              ldmatrix_x4(a, sst + kHRope + swz(row, 2 * ks + (lane >> 4)));
  #pragma unroll
              for (int nt = 0; nt < 2; ++nt) {
                const uint2 bq = qr[(ks * 2 + nt) * 32 + lane];
                mma_bf16(S[0][nt], a, bq.x, bq.y);
              }
            }
          }
        }

        // The team's last read of this stage: the code scales the value warps need (groups
        // 2tq, 2tq + 1 of this lane's four tokens) move to registers, and the stage is
        // released to the producer before the softmax.
        uint32_t kept_scl[2][2] = {{0u, 0u}, {0u, 0u}};
        if (cold && !kF8) {  // (float8 chunks have no scales)
          const uint16_t* scl = reinterpret_cast<const uint16_t*>(st + kScales);
#pragma unroll
          for (int m = 0; m < kCM; ++m)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int tk = ctok(m, gid + 8 * h);
              kept_scl[m][h] = (tk < t.n) ? *reinterpret_cast<const uint32_t*>(scl + 8 * tk + 2 * tq) : 0u;
            }
        }
        mbar_arrive(bar(kBarEmpty + s));

        // ---- finalize scores, mask, tile max ----
        const int n_m = cold ? kCM : 1;  // m-tiles of this tile's scores
        float tmax[2][2];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) tmax[nt][cc] = -INFINITY;
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const int h = c >> 1, cc = c & 1;
              const int r = 8 * nt + 2 * tq + cc;
              const int tk = cold ? ctok(m, gid + 8 * h) : 8 * tw + gid;
              bool valid = (m < n_m) && (cold || h == 0) && tk < t.n;
              if (t.kind == ASTERQ_TILE_NEW) valid = valid && (t.off + tk) <= (rb * kRows + r) / H;
              float sv = S[m][nt][c] * ((cold && !kF8) ? qinvi[nt][cc] : qinv[nt][cc]);
              if (p.logit_softcap > 0.0f) sv = p.logit_softcap * tanhf(sv / p.logit_softcap);
              sv = valid ? sv : -INFINITY;
              S[m][nt][c] = sv;
              tmax[nt][cc] = fmaxf(tmax[nt][cc], sv);
            }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int cc = 0; cc < 2; ++cc)
#pragma unroll
            for (int off = 4; off < 32; off <<= 1)
              tmax[nt][cc] = fmaxf(tmax[nt][cc], __shfl_xor_sync(0xffffffffu, tmax[nt][cc], off));
        float* wmax = misc + kMWmax + team * 128 + ((i >> 1) & 1) * 64;
        if (gid == 0) {
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) wmax[tw * 16 + 8 * nt + 2 * tq + cc] = tmax[nt][cc];
        }
        named_sync(1 + team, 32 * kTeamWarps);
        // the running max before this tile, published by the other team
        if (i > 0) mbar_wait(bar(kBarM), (i - 1) & 1, abort_flag, wait_limit(p));
        const float* m_in = misc + kMMrun + ((i - 1) & 1) * 16;
        float alpha_r[2][2], msub[2][2], lfac[2][2];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const int r = 8 * nt + 2 * tq + cc;
            const float mt = fmaxf(fmaxf(wmax[r], wmax[16 + r]), fmaxf(wmax[32 + r], wmax[48 + r]));
            const float m_prev = (i > 0) ? m_in[r] : -INFINITY;
            const float m_new = fmaxf(m_prev, mt);
            if (m_new == -INFINITY) {
              alpha_r[nt][cc] = 1.0f;
              msub[nt][cc] = 0.0f;
            } else {
              alpha_r[nt][cc] = ex2_ftz((m_prev - m_new) * kLog2e);
              msub[nt][cc] = m_new;
            }
            lfac[nt][cc] = (m_team[nt][cc] == -INFINITY) ? 0.0f : ex2_ftz((m_team[nt][cc] - m_new) * kLog2e);
            m_team[nt][cc] = m_new;
          }
        // publish the running max after tile i (lanes gid 0 of the team's first warp hold all
        // 16 rows).  Every thread of the team arrives once it has read the max before this
        // tile: the phase completes only then, so the other team cannot overwrite that slot
        // (with the max after tile i + 1) while a slow warp of this team still reads it.
        if (tw == 0 && gid == 0) {
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) misc[kMMrun + (i & 1) * 16 + 8 * nt + 2 * tq + cc] = m_team[nt][cc];
        }
        mbar_arrive(bar(kBarM));
        // ---- p = exp(s - m), handed to the value warps ----
        if (i >= 2) mbar_wait(bar(kBarPEmpty + b), ((i >> 1) - 1) & 1, abort_flag, wait_limit(p));
        float psum[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
        if (cold) {
          // p as fp16 [token][16 rows]; the two 16-byte halves of a token's row swap on every
          // other group of 4 tokens so that ldmatrix reads of 8 consecutive tokens hit 32 banks
          uint8_t* Pc = smem + kOffP + b * kPBytes;
          uint16_t* sT = reinterpret_cast<uint16_t*>(smem + kOffST + b * 2048);
#pragma unroll
          for (int m = 0; m < kCM; ++m)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int tk = ctok(m, gid + 8 * h);
#pragma unroll
              for (int nt = 0; nt < 2; ++nt) {
                const float p0 = ex2_ftz((S[m][nt][2 * h] - msub[nt][0]) * kLog2e);
                const float p1 = ex2_ftz((S[m][nt][2 * h + 1] - msub[nt][1]) * kLog2e);
                psum[nt][0] += p0;
                psum[nt][1] += p1;
                *reinterpret_cast<uint32_t*>(Pc + tk * 32 + ((nt ^ ((tk >> 2) & 1)) << 4) + 4 * tq) = pack_half2(p0, p1);
              }
              // lane tq publishes groups 2tq and 2tq + 1 of this token's code scales (0 outside the tile)
              sT[(2 * tq) * kColdTile + tk] = (uint16_t)(kept_scl[m][h] & 0xffffu);
              sT[(2 * tq + 1) * kColdTile + tk] = (uint16_t)(kept_scl[m][h] >> 16);
            }
        } else {
          float* P = reinterpret_cast<float*>(smem + kOffP + b * kPBytes);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              const float pv = ex2_ftz((S[0][nt][c] - msub[nt][c]) * kLog2e);
              P[(8 * nt + 2 * tq + c) * kPStride + 8 * tw + gid] = pv;
              psum[nt][c] += pv;
            }
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) psum[nt][cc] += __shfl_xor_sync(0xffffffffu, psum[nt][cc], off);
            l_w[nt][cc] = l_w[nt][cc] * lfac[nt][cc] + psum[nt][cc];
          }
        if (tw == 0 && gid == 0) {
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) misc[kMAlpha + b * 16 + 8 * nt + 2 * tq + cc] = alpha_r[nt][cc];
        }
        mbar_arrive(bar(kBarPFull + b));
      }
      // final per-warp sums, brought to the final running max, and the running max itself
      // (the team that did not take the last tile reads it from the other team: phase n_t - 1)
      const int last = n_t - 1;
      if (n_t > 0 && (last & 1) != team) mbar_wait(bar(kBarM), last & 1, abort_flag, wait_limit(p));
      named_sync(1 + team, 32 * kTeamWarps);
      if (gid == 0) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const int r = 8 * nt + 2 * tq + cc;
            const float m_fin = (n_t > 0) ? misc[kMMrun + (last & 1) * 16 + r] : -INFINITY;
            const float f = (m_team[nt][cc] == -INFINITY) ? 0.0f : exp2f((m_team[nt][cc] - m_fin) * kLog2e);
            misc[kMLw + warp * 16 + r] = l_w[nt][cc] * f;
            if (warp == 0) misc[kMWmax + r] = m_fin;
          }
      }
      named_sync(0, kThreads);
      if (epilogue()) break;
    }
  } else {
    // =====================================================================
    // value warps: scale group g = warp - 8, latent dims [64g, 64g + 64)
    // =====================================================================
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kBytes ? kValueRegsB : kValueRegs));
    const int g = warp - kScoreWarps;
    const bool rotated = p.cold_scheme == ASTERQ_SCHEME_HADAMARD_INT4;  // else plain int4: no rotation back
#pragma unroll 1
    for (int it = it_begin; it < it_end; ++it) {
      begin_item(it);
      if (it > it_begin) next_item_sync();
      if (warp == kProducerWarp) {
        if (lane == 0) prologue(it == it_begin);
        __syncwarp();
      }
      float o[4][2][4];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int d = 0; d < 4; ++d) o[a][c][d] = 0.0f;
      // order 0: accumulator holds cold tokens, rotated basis, code-derived row order
      // order 1: plain basis, natural row order
      int order = 1;
      if (n_t > 0) order = (load_tile(p, tile_begin).kind == ASTERQ_TILE_COLD) ? 0 : 1;
      // [16][512] scratch, usable once the cold query fragments are no longer read
      float* scratch_o = reinterpret_cast<float*>(smem + kOffQi);
      const int region = (g < 4) ? kCodesLo : kCodesHi;
      const int cchunk = 2 * (g & 3) + (gid >> 2);

      auto store_o = [&]() {
#pragma unroll
        for (int mi = 0; mi < 4; ++mi)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              // order 0, INT4: rows gid / gid + 8 of m-tile mi are dims 2(4gid + mi) / + 1 of the group;
              // int8: dims 8gid + mi / 8gid + 4 + mi
              const int dim = (order == 0) ? (kBytes ? 64 * g + 8 * gid + 4 * (c >> 1) + mi : 64 * g + 2 * (4 * gid + mi) + (c >> 1))
                                           : 64 * g + 16 * mi + gid + 8 * (c >> 1);
              scratch_o[(8 * nt + 2 * tq + (c & 1)) * kL + dim] = o[mi][nt][c];
            }
      };

      Tile t_next = (n_t > 0) ? load_tile(p, tile_begin) : Tile{ASTERQ_TILE_HOT, 0, 0, 0};
      int4 raw_next = (n_t > 1) ? fetch_tile(p, tile_begin + 1) : make_int4(0, 0, 0, 0);
      // producer lane: raw descriptor of the next tile it will issue
      int4 praw = (warp == kProducerWarp && lane == 0 && kStages < n_t) ? fetch_tile(p, tile_begin + kStages)
                                                                           : make_int4(0, 0, 0, 0);
#pragma unroll 1
      for (int i = 0; i < n_t; ++i) {
        const int s = i % kStages, b = i & 1;
        const Tile t = t_next;
        if (i + 1 < n_t) t_next = check_tile(p, raw_next);
        if (i + 2 < n_t) raw_next = fetch_tile(p, tile_begin + i + 2);
        mbar_wait(bar(kBarFull + i % kFullBars), (i / kFullBars) & 1, abort_flag, wait_limit(p));  // TMA data visible to this warp
        const uint8_t* st = smem + s * kStageBytes;
        const uint32_t sst = sbase + s * kStageBytes;
        const float* P = reinterpret_cast<const float*>(smem + kOffP + b * kPBytes);
        const bool cold = t.kind == ASTERQ_TILE_COLD;

        // This warp's whole share of the stage goes to registers first (cold: its code words
        // of all 128 tokens; hot: its bf16 A fragments of all 32 tokens), so the stage is
        // released, and refilled with tile i + 3, before this tile's p is even ready.
        uint32_t xs[8][4];
        if (cold && kBytes) {
          // int8: 8 bytes (dims 64g + 8gid .. + 7) of each of the lane's four tokens per k-step:
          // token j of k-step kt -> xs[2kt + (j >> 1)][2(j & 1) .. + 1]
#pragma unroll
          for (int kt = 0; kt < kColdTile8 / 16; ++kt) {
            const int t0 = 16 * kt + 2 * tq;
            const int tk[4] = {t0, t0 + 1, t0 + 8, t0 + 9};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint2 w = *reinterpret_cast<const uint2*>(st + (g >> 1) * kCodeBlock8 +
                                                         swz(tk[j], 4 * (g & 1) + (gid >> 1)) + 8 * (gid & 1));
              // rows past the tile's tokens hold whatever follows in the pool: any int8 byte is a
              // finite value that p = 0 cancels, but an e4m3 byte may be NaN (0 x NaN poisons the sum)
              if (kF8 && tk[j] >= t.n) w = make_uint2(0u, 0u);
              xs[2 * kt + (j >> 1)][2 * (j & 1)] = w.x;
              xs[2 * kt + (j >> 1)][2 * (j & 1) + 1] = w.y;
            }
          }
        } else if (cold) {
#pragma unroll
          for (int kt = 0; kt < kColdTile / 16; ++kt) {
            const int t0 = 16 * kt + 2 * tq;
            const int tk[4] = {t0, t0 + 1, t0 + 8, t0 + 9};  // this lane's k indices
#pragma unroll
            for (int j = 0; j < 4; ++j)
              xs[kt][j] = *reinterpret_cast<const uint32_t*>(st + region + swz(tk[j], cchunk) + 4 * (gid & 3));
          }
        } else {
          // rows beyond n hold stale data: zero this warp's latent block there
          // (p is 0 for them, but 0 x NaN would poison the accumulator)
          if (t.n < kHotTile) {
            for (int e = lane; e < (kHotTile - t.n) * 8; e += 32)
              *reinterpret_cast<uint4*>(smem + s * kStageBytes + g * kHotBlock + (t.n + e / 8) * 128 + (e % 8) * 16) =
                  make_uint4(0u, 0u, 0u, 0u);
            __syncwarp();
          }
#pragma unroll
          for (int kt = 0; kt < kHotTile / 16; ++kt)
#pragma unroll
            for (int mi = 0; mi < 4; ++mi) {
              const int row = 16 * kt + (lane & 7) + 8 * (lane >> 4);
              ldmatrix_x4_trans(xs[4 * kt + mi], sst + g * kHotBlock + swz(row, 2 * mi + ((lane >> 3) & 1)));
            }
          fence_async_shared();  // the zero fill precedes the next TMA write of this stage
        }
        mbar_arrive(bar(kBarEmpty + s));
        if (warp == kProducerWarp) {
          // refill this stage with tile i + 3 once the tile's team and every value warp have
          // released it; its descriptor was fetched a tile ago, so the issue does not wait
          // on global memory
          if (lane == 0 && i + kStages < n_t && mbar_wait(bar(kBarEmpty + s), (i / kStages) & 1, abort_flag, wait_limit(p)))
            issue_tile(i + kStages, check_tile(p, praw));
          if (lane == 0 && i + kStages + 1 < n_t) praw = fetch_tile(p, tile_begin + i + kStages + 1);
          __syncwarp();
        }
        mbar_wait(bar(kBarPFull + b), (i >> 1) & 1, abort_flag, wait_limit(p));

        if (!cold && order == 0) {
          // first hot tile after cold ones: rotate the accumulator back (O = H O_rot)
          store_o();
          named_sync(3, 32 * kValueWarps);
          if (rotated) {
            warp_fwht_rows(scratch_o, 2 * g, 2, lane);
            named_sync(3, 32 * kValueWarps);
          }
          order = 1;
#pragma unroll
          for (int mi = 0; mi < 4; ++mi)
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
              for (int c = 0; c < 4; ++c)
                o[mi][nt][c] = scratch_o[(8 * nt + 2 * tq + (c & 1)) * kL + 64 * g + 16 * mi + gid + 8 * (c >> 1)];
        }
        {
          float al[2][2];
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            al[nt][0] = misc[kMAlpha + b * 16 + 8 * nt + 2 * tq];
            al[nt][1] = misc[kMAlpha + b * 16 + 8 * nt + 2 * tq + 1];
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
          const uint32_t pbase = sbase + kOffP + b * kPBytes;
          const uint16_t* sT = reinterpret_cast<const uint16_t*>(smem + kOffST + b * 2048) + g * kColdTile;
          const int lt = (lane & 7) + 8 * ((lane >> 3) & 1), lhalf = lane >> 4;
#pragma unroll
          for (int kt = 0; kt < kCT / 16; ++kt) {
            // tokens 16kt + {2tq, 2tq+1, 2tq+8, 2tq+9} are this lane's k indices
            const int t0 = 16 * kt + 2 * tq;
            // p B fragments (fp16) of rows 0-7 / 8-15, times the tokens' group-g code scales
            uint32_t pr[4];
            {
              const int tok = 16 * kt + lt;
              ldmatrix_x4_trans(pr, pbase + tok * 32 + ((lhalf ^ ((tok >> 2) & 1)) << 4));
            }
            const uint32_t s01 = *reinterpret_cast<const uint32_t*>(sT + t0);
            const uint32_t s89 = *reinterpret_cast<const uint32_t*>(sT + t0 + 8);
            uint32_t pb[2][2];
            if constexpr (kF8) {  // float8 chunks have no scales
              pb[0][0] = pr[0];
              pb[0][1] = pr[1];
              pb[1][0] = pr[2];
              pb[1][1] = pr[3];
            } else {
              pb[0][0] = hmul2_u32(pr[0], s01);
              pb[0][1] = hmul2_u32(pr[1], s89);
              pb[1][0] = hmul2_u32(pr[2], s01);
              pb[1][1] = hmul2_u32(pr[3], s89);
            }
            if constexpr (kF8) {
#pragma unroll
              for (int mi = 0; mi < 4; ++mi) {
                // as for int8 below, with the byte pair (token t0, t0 + 1) in bits 0-15 converted
                // from e4m3 to fp16 (the low byte to the low half)
                const uint32_t sel = (uint32_t)mi | ((uint32_t)(4 + mi) << 4);
                const uint32_t* x01 = xs[2 * kt];
                const uint32_t* x89 = xs[2 * kt + 1];
                uint32_t a[4];
                a[0] = e4m3x2_to_f16x2(prmt(x01[0], x01[2], sel));
                a[1] = e4m3x2_to_f16x2(prmt(x01[1], x01[3], sel));
                a[2] = e4m3x2_to_f16x2(prmt(x89[0], x89[2], sel));
                a[3] = e4m3x2_to_f16x2(prmt(x89[1], x89[3], sel));
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) mma_f16(o[mi][nt], a, pb[nt][0], pb[nt][1]);
              }
            } else if constexpr (kB8) {
#pragma unroll
              for (int mi = 0; mi < 4; ++mi) {
                // rows gid / gid+8 of m-tile mi are dims 8gid + mi / 8gid + 4 + mi of group g: byte mi
                // of word 0 / word 1 of each token; a pair = the same byte of tokens (t0, t0 + 1)
                // in a[0], a[1] and (t0 + 8, t0 + 9) in a[2], a[3]
                const uint32_t sel = (uint32_t)mi | ((uint32_t)(4 + mi) << 8);
                const uint32_t* x01 = xs[2 * kt];
                const uint32_t* x89 = xs[2 * kt + 1];
                uint32_t a[4];
                a[0] = s8_bytes02_f16x2(prmt(x01[0], x01[2], sel));
                a[1] = s8_bytes02_f16x2(prmt(x01[1], x01[3], sel));
                a[2] = s8_bytes02_f16x2(prmt(x89[0], x89[2], sel));
                a[3] = s8_bytes02_f16x2(prmt(x89[1], x89[3], sel));
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) mma_f16(o[mi][nt], a, pb[nt][0], pb[nt][1]);
              }
            } else {
#pragma unroll
              for (int mi = 0; mi < 4; ++mi) {
                // rows gid / gid+8 of m-tile mi are dims 2(4gid+mi) / 2(4gid+mi)+1 of group g
                const uint32_t sel =
                    (uint32_t)mi | ((uint32_t)mi << 4) | ((uint32_t)(4 + mi) << 8) | ((uint32_t)(4 + mi) << 12);
                const uint32_t z01 = prmt(xs[kt][0], xs[kt][1], sel);
                const uint32_t z23 = prmt(xs[kt][2], xs[kt][3], sel);
                uint32_t a[4];
                a[0] = nib_lo_f16x2(z01);
                a[1] = nib_hi_f16x2(z01);
                a[2] = nib_lo_f16x2(z23);
                a[3] = nib_hi_f16x2(z23);
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) mma_f16(o[mi][nt], a, pb[nt][0], pb[nt][1]);
              }
            }
          }
        } else {
#pragma unroll
          for (int kt = 0; kt < kHotTile / 16; ++kt) {
            uint32_t pb[2][2][2];  // [ntile][hi/lo][b0/b1]
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
              const float2 p01 = *reinterpret_cast<const float2*>(P + (8 * nt + gid) * kPStride + 16 * kt + 2 * tq);
              const float2 p89 = *reinterpret_cast<const float2*>(P + (8 * nt + gid) * kPStride + 16 * kt + 2 * tq + 8);
              const uint32_t h0 = pack_bf162(p01.x, p01.y), h1 = pack_bf162(p89.x, p89.y);
              const float2 r0 = unpack_bf162(h0), r1 = unpack_bf162(h1);
              pb[nt][0][0] = h0;
              pb[nt][0][1] = h1;
              pb[nt][1][0] = pack_bf162(p01.x - r0.x, p01.y - r0.y);
              pb[nt][1][1] = pack_bf162(p89.x - r1.x, p89.y - r1.y);
            }
#pragma unroll
            for (int hl = 0; hl < 2; ++hl)
#pragma unroll
              for (int mi = 0; mi < 4; ++mi)
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) mma_bf16(o[mi][nt], xs[4 * kt + mi], pb[nt][hl][0], pb[nt][hl][1]);
          }
        }
        mbar_arrive(bar(kBarPEmpty + b));
      }
      // accumulator -> scratch in natural order, rotated back if it is still rotated.  The
      // scratch is the query-fragment region: an item with no tiles (a context-parallel
      // rank that holds none of a block's pages) waits for its query copy to land first,
      // or the copy could overwrite the zero record after it is stored.
      if (n_t == 0) mbar_wait(bar(kBarQ), 0, abort_flag, wait_limit(p));
      store_o();
      named_sync(3, 32 * kValueWarps);
      if (order == 0 && rotated) {
        warp_fwht_rows(scratch_o, 2 * g, 2, lane);
        named_sync(3, 32 * kValueWarps);
      }
      named_sync(0, kThreads);
      if (epilogue()) break;
    }
    // After a timed-out wait: the copies this CTA requested and nobody waited for land before
    // the CTA exits (bounded), so no copy writes into the shared memory of a later CTA.
    if (warp == kProducerWarp && lane == 0 && *abort_flag) {
      const int hi = *issued_hi;
      for (int j = max(0, hi - kStages); j < hi; ++j)
        for (int k = 0; k < (1 << 20) && !mbar_try(bar(kBarFull + j % kFullBars), (j / kFullBars) & 1); ++k) {
        }
    }
  }
}

// Merge partial records (latent_attention.py:212-220 applied across splits).
// Grid: (combine job, 4-dim slice of the latent), so a long sequence's many records are
// read by 128 CTAs per job.  256 threads: first the per-row max and sum over all of the
// job's records (16 threads per row, four records' loads in flight), then each (row,
// 4 dims) output is accumulated by 16 lanes that take every 16th record, four records'
// loads in flight per lane, and summed with shuffles.  The records' weights w / l are
// staged in shared memory 256 records at a time.  The loop is a chain of dependent L2
// round trips, so it is cut short by spreading records over lanes and CTAs.
constexpr int kCombDims = 4;
constexpr int kCombLanes = 16;        // record lanes per output
constexpr int kCombThreads = 256;     // 16 rows x 16 record lanes (one float4 of output each)
constexpr int kCombWindow = 256;      // records whose weights are staged at a time
// kMerge: write the merged record unnormalized (o, m, l) to record blockIdx.x of `out`
// (laid out like the workspace: o [n_jobs][16][latent_dim], m [n_jobs][16], l [n_jobs][16])
// instead of the normalized output rows.
// Where slot q of job j lives (floats): o rows at wo + j * o_job + q * o_slot + row * latent_dim,
// m at wm + j * ml_job + q * ml_slot + row (l likewise).  The workspace layout is
// {16 * latent_dim, 16, 0, 0}; records gathered rank-major from `world` ranks of `n`
// merged records each are {n * record, n * record, 16 * latent_dim, 16}, record = 16 * (latent_dim + 2).
struct SlotLayout {
  int64_t o_slot, ml_slot, o_job, ml_job;
};

template <bool kMerge>
__device__ __forceinline__ void combine_job(const float* __restrict__ wo, const float* __restrict__ wm,
                                            const float* __restrict__ wl, const int32_t* __restrict__ jobs, int n_slots,
                                            int n_jobs, int latent_dim, void* __restrict__ out, int out_dtype,
                                            const SlotLayout lay) {
  __shared__ float w_s[kCombWindow * kRows];
  __shared__ float row_s[2 * kRows];  // per-row max, 1 / sum
  wo += blockIdx.x * lay.o_job;
  wm += blockIdx.x * lay.ml_job;
  wl += blockIdx.x * lay.ml_job;
  const int4 job = *reinterpret_cast<const int4*>(jobs + 4 * (int64_t)blockIdx.x);
  const int slot_begin = max(job.x, 0), slot_end = min(job.y, n_slots), n_rows = min(job.w, kRows);
  const int64_t out_row0 = job.z;
  const int tid = threadIdx.x;
  if (!kMerge && slot_end <= slot_begin) return;  // (a merge still writes an empty record)
  {
    const int r = tid >> 4, j = tid & 15;
    float mmax = -INFINITY;
#pragma unroll 4
    for (int q = slot_begin + j; q < slot_end; q += 16) mmax = fmaxf(mmax, wm[q * lay.ml_slot + r]);
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffffu, mmax, off));
    const float msub = (mmax == -INFINITY) ? 0.0f : mmax;
    float l = 0.0f;
#pragma unroll 4
    for (int q = slot_begin + j; q < slot_end; q += 16)
      l += exp2f((wm[q * lay.ml_slot + r] - msub) * kLog2e) * wl[q * lay.ml_slot + r];
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    if (j == 0) {
      row_s[r] = msub;
      row_s[kRows + r] = kMerge ? 1.0f : 1.0f / fmaxf(l, 1e-20f);
      if (kMerge && blockIdx.y == 0) {
        float* mm = reinterpret_cast<float*>(out) + (int64_t)n_jobs * kRows * latent_dim;
        mm[(int64_t)blockIdx.x * kRows + r] = mmax;
        mm[(int64_t)n_jobs * kRows + (int64_t)blockIdx.x * kRows + r] = l;
      }
    }
  }
  const int lq = tid & (kCombLanes - 1), r = tid >> 4;
  const int d = blockIdx.y * kCombDims;
  float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (int w0 = slot_begin; w0 < slot_end; w0 += kCombWindow) {
    const int nw = min(kCombWindow, slot_end - w0);
    __syncthreads();  // row scalars written / previous window consumed
    for (int e = tid; e < nw * kRows; e += kCombThreads) {
      const int q = e >> 4, rr = e & 15;
      w_s[e] = exp2f((wm[(w0 + q) * lay.ml_slot + rr] - row_s[rr]) * kLog2e) * row_s[kRows + rr];
    }
    __syncthreads();
    int q = lq;
    for (; q + 3 * kCombLanes < nw; q += 4 * kCombLanes) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        v[u] = *reinterpret_cast<const float4*>(wo + (w0 + q + kCombLanes * u) * lay.o_slot + r * latent_dim + d);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float w = w_s[(q + kCombLanes * u) * kRows + r];
        acc.x += w * v[u].x;
        acc.y += w * v[u].y;
        acc.z += w * v[u].z;
        acc.w += w * v[u].w;
      }
    }
    for (; q < nw; q += kCombLanes) {
      const float4 v = *reinterpret_cast<const float4*>(wo + (w0 + q) * lay.o_slot + r * latent_dim + d);
      const float w = w_s[q * kRows + r];
      acc.x += w * v.x;
      acc.y += w * v.y;
      acc.z += w * v.z;
      acc.w += w * v.w;
    }
  }
#pragma unroll
  for (int off = 1; off < kCombLanes; off <<= 1) {
    acc.x += __shfl_xor_sync(0xffffffffu, acc.x, off);
    acc.y += __shfl_xor_sync(0xffffffffu, acc.y, off);
    acc.z += __shfl_xor_sync(0xffffffffu, acc.z, off);
    acc.w += __shfl_xor_sync(0xffffffffu, acc.w, off);
  }
  if (lq != 0 || d >= latent_dim) return;
  if (kMerge) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + ((int64_t)blockIdx.x * kRows + r) * latent_dim + d) = acc;
    return;
  }
  if (r >= n_rows) return;
  const int64_t off = (out_row0 + r) * latent_dim + d;
  if (out_dtype == ASTERQ_DTYPE_F32) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + off) = acc;
  } else {
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(out) + off) =
        make_uint2(pack_bf162(acc.x, acc.y), pack_bf162(acc.z, acc.w));
  }
}

__global__ void __launch_bounds__(kCombThreads) combine_kernel(const float* __restrict__ wo, const float* __restrict__ wm,
                                                      const float* __restrict__ wl, const int32_t* __restrict__ jobs,
                                                      int n_slots, int latent_dim, void* __restrict__ out,
                                                      int out_dtype, const SlotLayout lay,
                                                      const int32_t* __restrict__ n_live) {
  if (n_live != nullptr && (int)blockIdx.x >= __ldg(n_live)) return;  // beyond a device-built schedule's jobs
  combine_job<false>(wo, wm, wl, jobs, n_slots, 0, latent_dim, out, out_dtype, lay);
}

// Merge partial records into fewer partial records (same rule, no normalisation):
// job j turns slots [slot_begin, slot_end) into record j of `merged`, laid out like
// the workspace (o [n_jobs][16][latent_dim], then m [n_jobs][16], then l [n_jobs][16]).
// Context-parallel decode merges each rank's split-KV records this way before
// the records of all ranks are gathered.
__global__ void __launch_bounds__(kCombThreads) merge_kernel(const float* __restrict__ wo, const float* __restrict__ wm,
                                                    const float* __restrict__ wl, const int32_t* __restrict__ jobs,
                                                    int n_slots, int n_jobs, int latent_dim, float* __restrict__ merged) {
  combine_job<true>(wo, wm, wl, jobs, n_slots, n_jobs, latent_dim, merged, ASTERQ_DTYPE_F32,
                    SlotLayout{(int64_t)kRows * latent_dim, kRows, 0, 0});
}

// ---------------------------------------------------------------------------
// Context-parallel record exchange by peer stores (no collective library)
// ---------------------------------------------------------------------------
// Every rank owns one mailbox in its own device memory, which the other ranks map through
// CUDA IPC.  Layout: a 256-byte header (step counter, CTAs done, one flag per source rank),
// then the records, [2 step parities][world source ranks][n_blocks merged records], each
// rank's part laid out as merge_kernel writes it (o [n][16][512], m [n][16], l [n][16]).
// A step is merge_push_kernel then combine_wait_kernel on each rank's stream:
//  * merge_push merges the rank's split-KV pieces into one record per 16-row block and stores
//    it into slot `rank` of every rank's mailbox (its own and, over NVLink, its peers'); the
//    last of its CTAs then raises flag `rank` in every mailbox to the step number (a release
//    store at system scope after system-scope fences of every CTA's stores);
//  * combine_wait reads the step number, waits (bounded) until every rank's flag in its own
//    mailbox has reached it, and combines the records of all ranks from its own memory.
// Steps alternate between two record parities, so a rank that runs one step ahead writes the
// other parity; it cannot run two steps ahead, because its own combine waits for every rank's
// push of the step in between, which each rank issues only after its previous combine.
constexpr int kMailHeaderBytes = 256;
constexpr int kMailMaxWorld = 56;
struct MailHeader {
  unsigned counter;  // steps completed (written by the last CTA of merge_push)
  unsigned done;     // CTAs of the current merge_push that finished their stores
  unsigned pad[6];
  unsigned flags[kMailMaxWorld];  // flag r: the last step whose records rank r has stored here
};
static_assert(sizeof(MailHeader) <= kMailHeaderBytes, "mailbox header");

__host__ __device__ inline int64_t mail_rank_floats(int n_blocks, int latent_dim) {
  return (int64_t)n_blocks * kRows * (latent_dim + 2);
}

ASTERQ_DEVICE unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
ASTERQ_DEVICE void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(kCombThreads) merge_push_kernel(const float* __restrict__ wo,
                                                         const float* __restrict__ wm,
                                                         const float* __restrict__ wl,
                                                         const int32_t* __restrict__ jobs, int n_slots, int n_jobs,
                                                         int latent_dim, void* const* __restrict__ mailboxes,
                                                         int world, int rank) {
  MailHeader* own = reinterpret_cast<MailHeader*>(mailboxes[rank]);
  // every CTA reads the counter before the last CTA of this launch advances it
  const unsigned step = *reinterpret_cast<volatile unsigned*>(&own->counter) + 1u;
  const int64_t part = mail_rank_floats(n_jobs, latent_dim);
  const int64_t rec_off = ((int64_t)(step & 1u) * world + rank) * part;  // floats past the header
  float* mine = reinterpret_cast<float*>(reinterpret_cast<char*>(own) + kMailHeaderBytes) + rec_off;
  combine_job<true>(wo, wm, wl, jobs, n_slots, n_jobs, latent_dim, mine, ASTERQ_DTYPE_F32,
                    SlotLayout{(int64_t)kRows * latent_dim, kRows, 0, 0});
  __syncthreads();  // this CTA's part of the record is in `mine`
  // the same part, into every peer's mailbox: o rows (16 x 4 dims) and, for the first dim
  // chunk, the rows' m and l
  const int tid = threadIdx.x;
  const int d = blockIdx.y * kCombDims;
  int64_t off = -1;
  if (tid < kRows && d < latent_dim) {
    off = ((int64_t)blockIdx.x * kRows + tid) * latent_dim + d;
  } else if (blockIdx.y == 0 && tid >= 32 && tid < 32 + 2 * kRows) {
    const int k = tid - 32;  // m of row k, then l of row k - 16
    off = (int64_t)n_jobs * kRows * latent_dim + (k >= kRows ? (int64_t)n_jobs * kRows : 0) +
          (int64_t)blockIdx.x * kRows + (k & (kRows - 1));
  }
  if (off >= 0) {
    const bool vec = tid < kRows;
    const float4 v4 = vec ? *reinterpret_cast<const float4*>(mine + off) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float v1 = vec ? 0.0f : mine[off];
    for (int r = 0; r < world; ++r) {
      if (r == rank) continue;
      float* dst = reinterpret_cast<float*>(reinterpret_cast<char*>(mailboxes[r]) + kMailHeaderBytes) + rec_off + off;
      if (vec)
        *reinterpret_cast<float4*>(dst) = v4;
      else
        *dst = v1;
    }
  }
  __threadfence_system();  // this CTA's stores (local and remote) before its arrival below
  __syncthreads();
  if (tid == 0) {
    const unsigned total = gridDim.x * gridDim.y;
    if (atomicAdd(&own->done, 1u) == total - 1u) {
      __threadfence_system();  // every CTA's stores (observed through `done`) before the flags
      own->done = 0u;
      for (int r = 0; r < world; ++r) st_release_sys(&reinterpret_cast<MailHeader*>(mailboxes[r])->flags[rank], step);
      own->counter = step;
    }
  }
}

__global__ void __launch_bounds__(kCombThreads) combine_wait_kernel(const void* __restrict__ mailbox, int world,
                                                           int n_jobs, const int32_t* __restrict__ jobs,
                                                           int latent_dim, void* __restrict__ out, int out_dtype,
                                                           long long limit, int32_t* __restrict__ status) {
  const MailHeader* h = reinterpret_cast<const MailHeader*>(mailbox);
  // the step merge_push (earlier on this stream) has just completed
  const unsigned step = *reinterpret_cast<const volatile unsigned*>(&h->counter);
  __shared__ int ready;
  if (threadIdx.x == 0) {
    int ok = 1;
    const long long t0 = clock64();
    for (int r = 0; r < world && ok; ++r) {
      while ((int)(ld_acquire_sys(&h->flags[r]) - step) < 0) {
        if (clock64() - t0 > limit) {
          ok = 0;
          break;
        }
        __nanosleep(256);
      }
    }
    ready = ok;
    if (!ok && status != nullptr) atomicExch(status, 1);
  }
  __syncthreads();
  if (!ready) return;  // a rank's records never arrived: the output is left unwritten
  const int64_t part = mail_rank_floats(n_jobs, latent_dim);
  const float* base = reinterpret_cast<const float*>(reinterpret_cast<const char*>(mailbox) + kMailHeaderBytes) +
                      (int64_t)(step & 1u) * world * part;
  const float* wm = base + (int64_t)n_jobs * kRows * latent_dim;
  const float* wl = wm + (int64_t)n_jobs * kRows;
  combine_job<false>(base, wm, wl, jobs, world, 0, latent_dim, out, out_dtype,
                     SlotLayout{part, part, (int64_t)kRows * latent_dim, kRows});
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
int validate(const asterq_decode_params* p) {
  if (!p) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: null params");
  if (p->latent_dim != kL || p->rope_dim != kRope || p->group_size != 64)
    return set_error(ASTERQ_ERR_UNSUPPORTED, "decode: geometry latent=%d rope=%d group=%d unsupported (512/64/64)",
                     p->latent_dim, p->rope_dim, p->group_size);
  if (p->n_heads <= 0) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: n_heads must be positive");
  if (p->page_tokens <= 0 || p->page_tokens % 16)
    return set_error(ASTERQ_ERR_UNSUPPORTED, "decode: page_tokens %d must be a positive multiple of 16",
                     p->page_tokens);
  if (p->out_dtype != ASTERQ_DTYPE_F32 && p->out_dtype != ASTERQ_DTYPE_BF16)
    return set_error(ASTERQ_ERR_UNSUPPORTED, "decode: out_dtype must be f32 or bf16");
  if (p->cold_scheme != ASTERQ_SCHEME_HADAMARD_INT4 && p->cold_scheme != ASTERQ_SCHEME_INT4 &&
      p->cold_scheme != ASTERQ_SCHEME_INT8 && p->cold_scheme != ASTERQ_SCHEME_FLOAT8)
    return set_error(ASTERQ_ERR_UNSUPPORTED, "decode: cold scheme %d unsupported (hadamard_int4, int4, int8 or float8)",
                     p->cold_scheme);
  if (p->n_items < 0 || p->n_tiles < 0 || p->n_combine < 0 || p->n_slots < 0)
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: negative table size");
  if (p->n_items > 0 && (!p->items || !p->tiles || !p->q_lat || !p->q_rope || !p->out))
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: null pointer");
  if (p->rope_scheme != ASTERQ_ROPE_BF16 && p->rope_scheme != ASTERQ_ROPE_QUANTIZED)
    return set_error(ASTERQ_ERR_UNSUPPORTED, "decode: rope scheme %d unsupported (bf16 or quantized)", p->rope_scheme);
  if (p->n_cold_pages > 0 && (!p->cold_codes || (!p->cold_scales && p->cold_scheme != ASTERQ_SCHEME_FLOAT8) || !p->cold_rope))
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: null cold pool");
  if (p->n_cold_pages > 0 && p->rope_scheme == ASTERQ_ROPE_QUANTIZED && p->cold_scheme != ASTERQ_SCHEME_FLOAT8 &&
      !p->cold_rope_scales)
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: quantized RoPE keys need cold_rope_scales");
  if (p->n_hot_pages > 0 && (!p->hot_latent || !p->hot_rope))
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: null hot pool");
  if (p->n_items > 0 && p->total_q > 0 && (!p->new_latent || !p->new_rope))
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: null new-token arrays");
  const void* aligned[] = {p->q_lat, p->q_rope, p->new_latent, p->new_rope, p->cold_codes, p->cold_scales,
                           p->cold_rope, p->hot_latent, p->hot_rope, p->tiles, p->items, p->combine, p->out,
                           p->workspace, p->cold_rope_scales};
  for (const void* ptr : aligned)
    if (reinterpret_cast<uintptr_t>(ptr) & 15)
      return set_error(ASTERQ_ERR_MISALIGNED, "decode: pointers must be 16-byte aligned");
  if (p->n_units < 0) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: negative unit count");
  if (p->n_workers < 0 || (p->n_workers > 0 && !p->workers))
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: a worker count needs a workers table");
  if (reinterpret_cast<uintptr_t>(p->workers) & 3)
    return set_error(ASTERQ_ERR_MISALIGNED, "decode: the workers table must be 4-byte aligned");
  if (p->n_items > 0 && (p->n_units == 0 || !p->units))
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: work items need a units table");
  if (reinterpret_cast<uintptr_t>(p->units) & 7)
    return set_error(ASTERQ_ERR_MISALIGNED, "decode: the units table must be 8-byte aligned");
  if (p->unit_jobs && (reinterpret_cast<uintptr_t>(p->unit_jobs) & 3))
    return set_error(ASTERQ_ERR_MISALIGNED, "decode: the unit_jobs table must be 4-byte aligned");
  if (p->n_combine_total < 0) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: negative combine job count");
  const int64_t need = (int64_t)p->n_slots * kRecordBytes +
                       (p->n_items > 0 ? (int64_t)p->n_units * kQPrepBytes + counter_bytes(p->n_units) : 0);
  if (need > 0 && (!p->workspace || p->workspace_bytes < need))
    return set_error(ASTERQ_ERR_WORKSPACE, "decode: workspace of %lld bytes < %lld needed",
                     (long long)p->workspace_bytes, (long long)need);
  return ASTERQ_OK;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 2-D byte tensor [rows][row_bytes] read in boxes of [box_rows][128 B] with the
// 128-byte swizzle.  With blocks > 1 the rows are blocks x 128 B and the map is 3-D
// (128 B, rows, blocks): one box [blocks][box_rows][128 B] lands block-major, the layout
// the kernel reads (each block a [box_rows][128 B] region), in one instruction.  An empty
// pool gets a map of one row of a valid buffer; the kernel never references it (tiles of
// that kind fail validation).
int make_map(CUtensorMap* map, const void* base, int64_t rows, int row_bytes, int box_rows, const void* dummy,
             int dummy_row_bytes, int blocks = 1) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(ASTERQ_ERR_CUDA, "decode: cuTensorMapEncodeTiled unavailable");
  if (!base || rows <= 0) {
    base = dummy;
    rows = 1;
    row_bytes = dummy_row_bytes;
  }
  CUresult r;
  if (blocks == 1) {
    cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1u, 1u};
    r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    if (row_bytes < 128 * blocks) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode: row of %d bytes < %d blocks", row_bytes, blocks);
    cuuint64_t dims[3] = {128u, (cuuint64_t)rows, (cuuint64_t)blocks};
    cuuint64_t strides[2] = {(cuuint64_t)row_bytes, 128u};
    cuuint32_t box[3] = {128u, (cuuint32_t)box_rows, (cuuint32_t)blocks};
    cuuint32_t estr[3] = {1u, 1u, 1u};
    r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return set_error(ASTERQ_ERR_CUDA, "decode: tensor map encoding failed (%d)", (int)r);
  return ASTERQ_OK;
}

}  // namespace dec
}  // namespace asterq

using namespace asterq;

extern "C" int64_t asterq_decode_workspace_bytes(const asterq_decode_params* p) {
  if (!p) return 0;
  return (int64_t)max(p->n_slots, 0) * dec::kRecordBytes + (int64_t)max(p->n_units, 0) * dec::kQPrepBytes +
         dec::counter_bytes(max(p->n_units, 0));
}

extern "C" int asterq_latent_decode(const asterq_decode_params* p, void* stream) {
  clear_error();
  int st = dec::validate(p);
  if (st != ASTERQ_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (p->n_items > 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    static unsigned long long configured = 0;  // one bit per device ordinal
    if (dev >= 64 || !(configured & (1ull << dev))) {
      const void* kernels[] = {reinterpret_cast<const void*>(dec::decode_kernel<dec::kModeInt4>),
                               reinterpret_cast<const void*>(dec::decode_kernel<dec::kModeInt4RopeQ>),
                               reinterpret_cast<const void*>(dec::decode_kernel<dec::kModeInt8>),
                               reinterpret_cast<const void*>(dec::decode_kernel<dec::kModeF8>),
                               reinterpret_cast<const void*>(dec::decode_kernel<dec::kModeInt8RopeQ>),
                               reinterpret_cast<const void*>(dec::decode_kernel<dec::kModeF8RopeQ>)};
      cudaError_t e = cudaSuccess;
      for (const void* fn : kernels)
        if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, dec::kSmemBytes);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(dec::qprep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dec::kPrepSmem);
      if (e != cudaSuccess) return set_error(ASTERQ_ERR_CUDA, "latent_decode: %s", cudaGetErrorString(e));
      // the score/value register split (setmaxnreg) assumes exactly kLaunchRegs per thread at launch:
      // refuse to launch a build that allocates fewer (an increase could then never be granted)
      for (const void* fn : kernels) {
        cudaFuncAttributes fa;
        e = cudaFuncGetAttributes(&fa, fn);
        if (e != cudaSuccess) return set_error(ASTERQ_ERR_CUDA, "latent_decode: %s", cudaGetErrorString(e));
        if (fa.numRegs != dec::kLaunchRegs)
          return set_error(ASTERQ_ERR_CUDA, "latent_decode: kernel built with %d registers per thread, the register split needs %d",
                           fa.numRegs, dec::kLaunchRegs);
      }
      if (dev < 64) configured |= (1ull << dev);
    }
    dec::TensorMaps maps;
    // q_lat rows are 1024 bytes (16 heads x 512 bf16 at least): a valid stand-in
    // base for the map of an empty pool
    const void* dummy = p->q_lat;
    const int64_t cold_rows = p->n_cold_pages * p->page_tokens, hot_rows = p->n_hot_pages * p->page_tokens;
    const bool b8 = p->cold_scheme == ASTERQ_SCHEME_INT8 || p->cold_scheme == ASTERQ_SCHEME_FLOAT8;  // byte codes
    const int ct = b8 ? dec::kColdTile8 : dec::kColdTile;
    if ((st = b8 ? dec::make_map(&maps.codes, p->cold_codes, cold_rows, 512, ct, dummy, 1024, 4)
                 : dec::make_map(&maps.codes, p->cold_codes, cold_rows, 256, ct, dummy, 1024, 2)) ||
        // (quantized RoPE codes come in by plain bulk copies: no tensor map over their pool)
        (st = dec::make_map(&maps.crope, p->rope_scheme == ASTERQ_ROPE_BF16 ? p->cold_rope : nullptr, cold_rows,
                            128, ct, dummy, 1024)) ||
        (st = dec::make_map(&maps.hlat, p->hot_latent, hot_rows, 1024, dec::kHotTile, dummy, 1024, 8)) ||
        (st = dec::make_map(&maps.hrope, p->hot_rope, hot_rows, 128, dec::kHotTile, dummy, 1024)) ||
        (st = dec::make_map(&maps.nlat, p->new_latent, p->total_q, 1024, dec::kHotTile, dummy, 1024, 8)) ||
        (st = dec::make_map(&maps.nrope, p->new_rope, p->total_q, 128, dec::kHotTile, dummy, 1024)))
      return st;
    dec::qprep_kernel<<<p->n_units, dec::kPrepThreads, dec::kPrepSmem, s>>>(*p);
    st = check_launch("latent_decode (query preparation)");
    if (st != ASTERQ_OK) return st;
    // with a workers table, one CTA per worker (the table is read only when n_workers > 0)
    asterq_decode_params kp = *p;
    if (kp.n_workers == 0) kp.workers = nullptr;
    const int grid = (kp.n_workers > 0) ? kp.n_workers : kp.n_items;
    if (grid > 0) {
      // programmatic dependent launch: the decode grid starts while qprep_kernel finishes
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(grid);
      cfg.blockDim = dim3(dec::kThreads);
      cfg.dynamicSmemBytes = dec::kSmemBytes;
      cfg.stream = s;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      const bool rq = kp.rope_scheme == ASTERQ_ROPE_QUANTIZED;
      cudaError_t e;
      if (kp.cold_scheme == ASTERQ_SCHEME_FLOAT8)
        e = rq ? cudaLaunchKernelEx(&cfg, dec::decode_kernel<dec::kModeF8RopeQ>, kp, maps)
               : cudaLaunchKernelEx(&cfg, dec::decode_kernel<dec::kModeF8>, kp, maps);
      else if (kp.cold_scheme == ASTERQ_SCHEME_INT8)
        e = rq ? cudaLaunchKernelEx(&cfg, dec::decode_kernel<dec::kModeInt8RopeQ>, kp, maps)
               : cudaLaunchKernelEx(&cfg, dec::decode_kernel<dec::kModeInt8>, kp, maps);
      else
        e = rq ? cudaLaunchKernelEx(&cfg, dec::decode_kernel<dec::kModeInt4RopeQ>, kp, maps)
               : cudaLaunchKernelEx(&cfg, dec::decode_kernel<dec::kModeInt4>, kp, maps);
      if (e != cudaSuccess) return set_error(ASTERQ_ERR_CUDA, "latent_decode: launch failed: %s", cudaGetErrorString(e));
    }
    st = check_launch("latent_decode");
    if (st != ASTERQ_OK) return st;
  }
  if (p->n_combine > 0) {
    const float* wo = reinterpret_cast<const float*>(p->workspace);
    const float* wm = wo + (int64_t)p->n_slots * dec::kRows * dec::kL;
    const float* wl = wm + (int64_t)p->n_slots * dec::kRows;
    dec::combine_kernel<<<dim3(p->n_combine, dec::kL / dec::kCombDims), dec::kCombThreads, 0, s>>>(
        wo, wm, wl, p->combine, p->n_slots, dec::kL, p->out, p->out_dtype,
        dec::SlotLayout{(int64_t)dec::kRows * dec::kL, dec::kRows, 0, 0},
        p->plan_counts != nullptr ? p->plan_counts + 6 : nullptr);
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
  if ((reinterpret_cast<uintptr_t>(partials) | reinterpret_cast<uintptr_t>(combine) | reinterpret_cast<uintptr_t>(out)) &
      15)
    return set_error(ASTERQ_ERR_MISALIGNED, "combine: pointers must be 16-byte aligned");
  const float* wm = partials + (int64_t)n_slots * dec::kRows * latent_dim;
  const float* wl = wm + (int64_t)n_slots * dec::kRows;
  dec::combine_kernel<<<dim3(n_combine, dec::kL / dec::kCombDims), dec::kCombThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      partials, wm, wl, combine, n_slots, latent_dim, out, out_dtype,
      dec::SlotLayout{(int64_t)dec::kRows * latent_dim, dec::kRows, 0, 0}, nullptr);
  return check_launch("splitkv_combine");
}

extern "C" int asterq_splitkv_merge(const float* partials, int32_t n_slots, const int32_t* jobs, int32_t n_jobs,
                                    int32_t latent_dim, float* merged, void* stream) {
  clear_error();
  if (latent_dim != dec::kL) return set_error(ASTERQ_ERR_UNSUPPORTED, "merge: latent_dim must be 512");
  if (n_slots < 0 || n_jobs < 0) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "merge: negative sizes");
  if (n_jobs == 0) return ASTERQ_OK;
  if (!partials || !jobs || !merged) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "merge: null pointer");
  if ((reinterpret_cast<uintptr_t>(partials) | reinterpret_cast<uintptr_t>(jobs) | reinterpret_cast<uintptr_t>(merged)) &
      15)
    return set_error(ASTERQ_ERR_MISALIGNED, "merge: pointers must be 16-byte aligned");
  const float* wm = partials + (int64_t)n_slots * dec::kRows * latent_dim;
  const float* wl = wm + (int64_t)n_slots * dec::kRows;
  dec::merge_kernel<<<dim3(n_jobs, dec::kL / dec::kCombDims), dec::kCombThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      partials, wm, wl, jobs, n_slots, n_jobs, latent_dim, merged);
  return check_launch("splitkv_merge");
}

extern "C" int asterq_splitkv_combine_ranks(const float* gathered, int32_t world, int32_t n_blocks,
                                            const int32_t* jobs, int32_t latent_dim, void* out, int32_t out_dtype,
                                            void* stream) {
  clear_error();
  if (latent_dim != dec::kL) return set_error(ASTERQ_ERR_UNSUPPORTED, "combine_ranks: latent_dim must be 512");
  if (world <= 0 || n_blocks < 0) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "combine_ranks: bad sizes");
  if (n_blocks == 0) return ASTERQ_OK;
  if (!gathered || !jobs || !out) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "combine_ranks: null pointer");
  if (out_dtype != ASTERQ_DTYPE_F32 && out_dtype != ASTERQ_DTYPE_BF16)
    return set_error(ASTERQ_ERR_UNSUPPORTED, "combine_ranks: out_dtype must be f32 or bf16");
  if ((reinterpret_cast<uintptr_t>(gathered) | reinterpret_cast<uintptr_t>(jobs) | reinterpret_cast<uintptr_t>(out)) &
      15)
    return set_error(ASTERQ_ERR_MISALIGNED, "combine_ranks: pointers must be 16-byte aligned");
  // rank r's part: o [n_blocks][16][512], m [n_blocks][16], l [n_blocks][16]
  const int64_t part = (int64_t)n_blocks * dec::kRows * (latent_dim + 2);
  const float* wm = gathered + (int64_t)n_blocks * dec::kRows * latent_dim;
  const float* wl = wm + (int64_t)n_blocks * dec::kRows;
  dec::combine_kernel<<<dim3(n_blocks, dec::kL / dec::kCombDims), dec::kCombThreads, 0,
                        reinterpret_cast<cudaStream_t>(stream)>>>(
      gathered, wm, wl, jobs, world, latent_dim, out, out_dtype,
      dec::SlotLayout{part, part, (int64_t)dec::kRows * latent_dim, dec::kRows}, nullptr);
  return check_launch("splitkv_combine_ranks");
}

extern "C" int64_t asterq_mailbox_bytes(int32_t world, int32_t n_blocks, int32_t latent_dim) {
  if (world < 1 || world > dec::kMailMaxWorld || n_blocks < 1 || latent_dim != dec::kL) return 0;
  return dec::kMailHeaderBytes + 2LL * world * dec::mail_rank_floats(n_blocks, latent_dim) * 4;
}

extern "C" int asterq_mailbox_create(int64_t bytes, void** dev_ptr, void* ipc_handle) {
  clear_error();
  if (bytes <= dec::kMailHeaderBytes || !dev_ptr || !ipc_handle)
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "mailbox_create: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e != cudaSuccess) return set_error(ASTERQ_ERR_CUDA, "mailbox_create: cudaMalloc: %s", cudaGetErrorString(e));
  e = cudaMemset(p, 0, (size_t)bytes);  // counter, done count and flags start at 0
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(p);
    return set_error(ASTERQ_ERR_CUDA, "mailbox_create: %s", cudaGetErrorString(e));
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == ASTERQ_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(ipc_handle, &h, sizeof(h));
  *dev_ptr = p;
  return ASTERQ_OK;
}

extern "C" int asterq_mailbox_open(const void* ipc_handle, void** peer_ptr) {
  clear_error();
  if (!ipc_handle || !peer_ptr) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "mailbox_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(ASTERQ_ERR_CUDA, "mailbox_open: %s", cudaGetErrorString(e));
  return ASTERQ_OK;
}

extern "C" int asterq_mailbox_close(void* peer_ptr) {
  clear_error();
  if (!peer_ptr) return ASTERQ_OK;
  cudaError_t e = cudaIpcCloseMemHandle(peer_ptr);
  if (e != cudaSuccess) return set_error(ASTERQ_ERR_CUDA, "mailbox_close: %s", cudaGetErrorString(e));
  return ASTERQ_OK;
}

extern "C" int asterq_mailbox_destroy(void* dev_ptr) {
  clear_error();
  if (!dev_ptr) return ASTERQ_OK;
  cudaError_t e = cudaFree(dev_ptr);
  if (e != cudaSuccess) return set_error(ASTERQ_ERR_CUDA, "mailbox_destroy: %s", cudaGetErrorString(e));
  return ASTERQ_OK;
}

extern "C" int asterq_cp_merge_push(const float* partials, int32_t n_slots, const int32_t* jobs, int32_t n_blocks,
                                    int32_t latent_dim, void* const* mailboxes, int32_t world, int32_t rank,
                                    void* stream) {
  clear_error();
  if (latent_dim != dec::kL) return set_error(ASTERQ_ERR_UNSUPPORTED, "merge_push: latent_dim must be 512");
  if (n_slots < 0 || n_blocks < 1 || world < 1 || world > dec::kMailMaxWorld || rank < 0 || rank >= world)
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "merge_push: bad sizes (world %d, rank %d, blocks %d)", world, rank,
                     n_blocks);
  if (!partials || !jobs || !mailboxes) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "merge_push: null pointer");
  if ((reinterpret_cast<uintptr_t>(partials) | reinterpret_cast<uintptr_t>(jobs) |
       reinterpret_cast<uintptr_t>(mailboxes)) & 15)
    return set_error(ASTERQ_ERR_MISALIGNED, "merge_push: pointers must be 16-byte aligned");
  const float* wm = partials + (int64_t)n_slots * dec::kRows * latent_dim;
  const float* wl = wm + (int64_t)n_slots * dec::kRows;
  dec::merge_push_kernel<<<dim3(n_blocks, dec::kL / dec::kCombDims), dec::kCombThreads, 0,
                           reinterpret_cast<cudaStream_t>(stream)>>>(partials, wm, wl, jobs, n_slots, n_blocks,
                                                                     latent_dim, mailboxes, world, rank);
  return check_launch("cp_merge_push");
}

extern "C" int asterq_cp_combine_wait(const void* mailbox, int32_t world, int32_t n_blocks, const int32_t* jobs,
                                      int32_t latent_dim, void* out, int32_t out_dtype, int64_t wait_limit_cycles,
                                      int32_t* status, void* stream) {
  clear_error();
  if (latent_dim != dec::kL) return set_error(ASTERQ_ERR_UNSUPPORTED, "combine_wait: latent_dim must be 512");
  if (world < 1 || world > dec::kMailMaxWorld || n_blocks < 1)
    return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "combine_wait: bad sizes");
  if (!mailbox || !jobs || !out) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "combine_wait: null pointer");
  if (out_dtype != ASTERQ_DTYPE_F32 && out_dtype != ASTERQ_DTYPE_BF16)
    return set_error(ASTERQ_ERR_UNSUPPORTED, "combine_wait: out_dtype must be f32 or bf16");
  if ((reinterpret_cast<uintptr_t>(mailbox) | reinterpret_cast<uintptr_t>(jobs) | reinterpret_cast<uintptr_t>(out)) & 15)
    return set_error(ASTERQ_ERR_MISALIGNED, "combine_wait: pointers must be 16-byte aligned");
  const long long limit = wait_limit_cycles > 0 ? wait_limit_cycles : kDefaultWaitLimit;
  dec::combine_wait_kernel<<<dim3(n_blocks, dec::kL / dec::kCombDims), dec::kCombThreads, 0,
                             reinterpret_cast<cudaStream_t>(stream)>>>(mailbox, world, n_blocks, jobs, latent_dim, out,
                                                                       out_dtype, limit, status);
  return check_launch("cp_combine_wait");
}

// ---------------------------------------------------------------------------
// Allocation-free entry point.
//
// Some callers cannot allocate device memory when they decode: a serving loop
// that pre-plans its memory and forbids allocator calls on the hot path, code
// that runs while a CUDA graph is being recorded elsewhere on the device, or a
// host runtime with no allocator of its own (a plain C caller that only receives
// pointers to its inputs and outputs).  For them the split-KV partial records
// live in a fixed array compiled into this library instead of a caller-provided
// workspace.  The array is a device global: every GPU that loads the library
// keeps it (room for kNoAllocMaxSlots partial records, kNoAllocMaxUnits
// prepared query blocks and one fused-combine counter per block, about 17.5 MB)
// until the process exits.  The array keeps the previous call's contents; the
// only part that must start at zero, the counters, is zeroed by the query
// preparation at the start of every call.
// ---------------------------------------------------------------------------
namespace asterq {
namespace dec {

constexpr int kNoAllocMaxSlots = 256;
constexpr int kNoAllocMaxUnits = 256;
static __device__ __align__(256) float
    g_noalloc_workspace[(kNoAllocMaxSlots * kRecordBytes + kNoAllocMaxUnits * kQPrepBytes + 4 * kNoAllocMaxUnits) / 4];

// the calling thread's current CUDA context (driver API, looked up through the runtime), or null
void* current_context() {
  using CtxGetCurrentFn = CUresult (*)(CUcontext*);
  static CtxGetCurrentFn fn = []() -> CtxGetCurrentFn {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<CtxGetCurrentFn>(f);
    return nullptr;
  }();
  CUcontext c = nullptr;
  if (fn && fn(&c) == CUDA_SUCCESS) return reinterpret_cast<void*>(c);
  return nullptr;
}

}  // namespace dec
}  // namespace asterq

extern "C" int asterq_latent_decode_noalloc(const asterq_decode_params* p, void* stream) {
  clear_error();
  if (!p) return set_error(ASTERQ_ERR_INVALID_ARGUMENT, "decode (no-alloc): null params");
  if (p->n_slots > dec::kNoAllocMaxSlots || p->n_units > dec::kNoAllocMaxUnits)
    return set_error(ASTERQ_ERR_WORKSPACE,
                     "decode (no-alloc): the schedule needs %d partial records and %d query blocks but the built-in "
                     "workspace holds %d and %d; build the plan with fewer split items or smaller batches, or call "
                     "asterq_latent_decode with a workspace",
                     p->n_slots, p->n_units, dec::kNoAllocMaxSlots, dec::kNoAllocMaxUnits);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(ASTERQ_ERR_CUDA, "decode (no-alloc): %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(ASTERQ_ERR_UNSUPPORTED, "decode (no-alloc): device ordinal %d >= 64", dev);
  // Host code cannot use g_noalloc_workspace's name as a device address: resolve it
  // with the device current, once per device and CUDA context (the first call on a
  // device does this, and the first call after the device's context changes, e.g.
  // after cudaDeviceReset reloaded the module; make those calls before any stream
  // capture).  The resolved address is remembered together with the context it
  // belongs to, under a lock.
  static std::mutex lock;
  static void* ctx_of[64] = {};
  static void* addr[64] = {};
  void* ctx = dec::current_context();
  void* ptr = nullptr;
  {
    std::lock_guard<std::mutex> guard(lock);
    if (!addr[dev] || ctx_of[dev] != ctx) {
      void* resolved = nullptr;
      e = cudaGetSymbolAddress(&resolved, dec::g_noalloc_workspace);
      if (e != cudaSuccess || !resolved)
        return set_error(ASTERQ_ERR_CUDA, "decode (no-alloc): cannot resolve the workspace address: %s",
                         cudaGetErrorString(e));
      addr[dev] = resolved;
      ctx_of[dev] = ctx;
    }
    ptr = addr[dev];
  }
  asterq_decode_params q = *p;
  q.workspace = ptr;
  q.workspace_bytes = (int64_t)sizeof(dec::g_noalloc_workspace);
  return asterq_latent_decode(&q, stream);
}
