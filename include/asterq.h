/*
 * asterq — B200 (sm_100a) kernels for AsterLM's Hadamard-INT4 latent-cache
 * global-attention decode.  Plain C ABI: device pointers, sizes and a CUDA
 * stream handle (passed as void*); no framework types.
 *
 * Reference interfaces each entry point replaces (AsterLM-Frontier, paths
 * relative to its project root):
 *   asterq_quantize        quantization/kv.py:76-118   quantize_tensor(x, scheme, group_size)
 *   asterq_dequantize      quantization/kv.py:121-134  dequantize_tensor(q, dtype)
 *   asterq_fwht            quantization/kv.py:13-32    normalized_fwht(x)
 *   asterq_latent_decode   layers/latent_attention.py:177-231 _absorbed_decode (q_len = 1) and
 *                          layers/latent_attention.py:116-175 _full_attention (q_len > 1, causal),
 *                          iterating the cache like cache.py:139-159 iter_chunks
 *   asterq_splitkv_combine layers/latent_attention.py:212-220 (the online-softmax merge rule)
 *   asterq_splitkv_merge   the same rule, leaving merged (m, l, o) records for a later combine
 *   asterq_cp_merge_push / asterq_cp_combine_wait  the same rule across ranks, records exchanged
 *                          by peer stores into CUDA IPC mailboxes (no counterpart: the
 *                          reference is single-device)
 *   asterq_splitkv_combine_ranks  the same rule over the merged records of all ranks, read where
 *                          a rank-major all-gather left them
 *
 * Every function returns ASTERQ_OK (0) or a negative status and never aborts;
 * asterq_last_error() describes the last failure on the calling thread.  All
 * work is enqueued on the given stream; nothing is allocated and nothing
 * synchronizes the host.
 */
#ifndef ASTERQ_H_
#define ASTERQ_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ASTERQ_VERSION 1

/* status codes */
#define ASTERQ_OK 0
#define ASTERQ_ERR_INVALID_ARGUMENT -1 /* bad shape, size or pointer (reference: ValueError) */
#define ASTERQ_ERR_UNSUPPORTED -2      /* valid request outside what the kernels implement */
#define ASTERQ_ERR_MISALIGNED -3       /* pointer or stride not aligned as required */
#define ASTERQ_ERR_WORKSPACE -4        /* workspace missing or too small */
#define ASTERQ_ERR_CUDA -5             /* CUDA launch error */

/* element types */
#define ASTERQ_DTYPE_F32 0
#define ASTERQ_DTYPE_BF16 1
#define ASTERQ_DTYPE_F16 2

/* storage schemes (kv.py:90 "int8", "int4", "hadamard_int4") */
#define ASTERQ_SCHEME_HADAMARD_INT4 0
#define ASTERQ_SCHEME_INT4 1
#define ASTERQ_SCHEME_INT8 2
#define ASTERQ_SCHEME_FLOAT8 3 /* kv.py:85-89 "float8": x.to(float8_e4m3fn), one byte a value, no scales */

/* cold RoPE keys (cache.py:160-164: quantized only with quantize_rope=True) */
#define ASTERQ_ROPE_BF16 0      /* cold_rope: bf16 [tokens][rope_dim] */
#define ASTERQ_ROPE_QUANTIZED 1 /* cold_rope: codes of the cold scheme, one scale group of rope_dim:
                                   [tokens][rope_dim/2] INT4 (Hadamard-rotated for hadamard_int4) or
                                   [tokens][rope_dim] int8 / float8 bytes; cold_rope_scales: fp16
                                   [tokens] (none for float8) */

/* tile kinds in the decode schedule */
#define ASTERQ_TILE_COLD 0 /* tokens of a cold page: INT4 (or int8) codes + fp16 scales + RoPE key */
#define ASTERQ_TILE_HOT 1  /* tokens of a hot page: bf16 latent + bf16 RoPE key */
#define ASTERQ_TILE_NEW 2  /* the step's own new tokens (causal among themselves) */
#define ASTERQ_TILE_HOLD 3 /* failure-detection test hook: nothing is loaded for this tile and its
                              arrival is never signalled, so the waits for it run into the bounded-wait
                              limit; the call then ends with *device_status = 1 and no output */

int asterq_version(void);
const char* asterq_last_error(void);

/*
 * Cache write path: rotate (hadamard_int4 only), groupwise absmax-quantize and
 * pack n_tokens rows of `dim` values.  Replaces quantize_tensor
 * (quantization/kv.py:76-118).  Output is bit-identical to the reference:
 *   codes  uint8 [n_tokens, P/2] (int4; P = padded width) or int8 [n_tokens, P]
 *   scales fp16  [n_tokens, P/group_size]
 * where P = next power of two >= dim for hadamard_int4 and
 * ceil(dim/group_size)*group_size otherwise.  x_dtype: ASTERQ_DTYPE_*.
 * x_row_stride is in elements.  P <= 512, group_size in {16, 32, 64}.
 * ASTERQ_SCHEME_FLOAT8: codes [n_tokens, dim] float8 e4m3 bytes as torch's
 * x.to(torch.float8_e4m3fn) writes them (round to nearest even, subnormals kept,
 * NaN, infinities and |x| > 464 become NaN with the sign of x); no scales (`scales`
 * and `group_size` are not used).
 */
int asterq_quantize(const void* x, int x_dtype, int64_t n_tokens, int dim, int64_t x_row_stride, int scheme,
                    int group_size, void* codes, void* scales, void* stream);

/*
 * Inverse of asterq_quantize (dequantize_tensor, quantization/kv.py:121-134):
 * codes * float(scale), inverse normalized FWHT for hadamard_int4, cropped to
 * `dim`, rounded to out_dtype.  Bit-identical to the reference.  ASTERQ_SCHEME_FLOAT8:
 * the e4m3 values widened to out_dtype (exact); `scales` is not used.
 */
int asterq_dequantize(const void* codes, const void* scales, int64_t n_tokens, int dim, int scheme, int group_size,
                      void* out, int out_dtype, int64_t out_row_stride, void* stream);

/* Normalized Walsh-Hadamard transform of float32 rows (kv.py:13-32), bit-exact; n in 2..512. */
int asterq_fwht(const float* x, float* y, int64_t rows, int n, void* stream);

/*
 * Health of the write path: *timeouts = how many encode warps gave up waiting
 * for a bulk copy of their input rows (each such wait is bounded at about two
 * seconds, after which the warp stops, so its rows' codes are not written).
 * Synchronizes the current device.  0 in normal operation.
 */
int asterq_codec_status(int32_t* timeouts);

/*
 * Decode attention over a paged hybrid latent cache.
 *
 * Layout in device memory (all row-major, token-major):
 *   cold_codes  uint8 [n_cold_pages, page_tokens, latent_dim/2]   rotated INT4 codes (kv.py:41-48 packing)
 *   cold_scales fp16  [n_cold_pages, page_tokens, latent_dim/64]
 *   cold_rope   bf16  [n_cold_pages, page_tokens, rope_dim]        (rope_scheme ASTERQ_ROPE_BF16), or
 *               uint8 [n_cold_pages, page_tokens, rope_dim/2]      (ASTERQ_ROPE_QUANTIZED: INT4 codes; int8 and
 *                                                                   float8: [.., rope_dim] bytes)
 *   cold_rope_scales fp16 [n_cold_pages, page_tokens]              (ASTERQ_ROPE_QUANTIZED only)
 *   hot_latent  bf16  [n_hot_pages, page_tokens, latent_dim]
 *   hot_rope    bf16  [n_hot_pages, page_tokens, rope_dim]
 *   q_lat       bf16  [total_q, n_heads, latent_dim]   absorbed query q_content @ W_k
 *   q_rope      bf16  [total_q, n_heads, rope_dim]     RoPE already applied
 *   new_latent  bf16  [total_q, latent_dim]            the step's own tokens (attended causally)
 *   new_rope    bf16  [total_q, rope_dim]
 *   out         [total_q, n_heads, latent_dim] in out_dtype: the context latent
 *               running_context / max(running_sum, 1e-20) (latent_attention.py:229)
 *
 * Schedule (built by the host, see the Python package's plan builder):
 *   tiles [n_tiles][4] int32 = {kind, page (ASTERQ_TILE_NEW: first new-token row), token offset, n_tokens}
 *          cold tiles hold <= 128 tokens (<= 64 with int8 codes), hot/new tiles <= 32 tokens; a tile
          never crosses a page.
 *   units [n_units][2] int32 = {out_row0, n_rows}: one per 16-row query block; its query operands
 *          (rotated, fixed-point, fragment-ordered) are prepared once per call into the workspace.
 *   items [n_items][8] int32 = {unit, row_block, tile_begin, tile_end, slot, out_row0, n_rows, q_len}
 *          16 query rows (t, h) per row block, rows flattened as t*n_heads + h; one CTA per item, or
 *          with a workers table one CTA per worker running its items in order.
 *          slot < 0: the item covers the whole sequence and writes `out` directly;
 *          slot >= 0: it writes an (m, l, o) partial to the workspace.
 *   combine [n_combine][4] int32 = {slot_begin, slot_end, out_row0, n_rows}: merges partials into `out`.
 * Cold schemes: hadamard_int4 and int4 (params.cold_scheme), and int8 (codes uint8/int8
 *   [n_cold_pages, page_tokens, latent_dim]: one signed byte a dim, kv.py scheme "int8",
 *   scales as above, not rotated), and float8 (e4m3 bytes [.., latent_dim], no scales: cold_scales
 *   may be NULL).
 * Geometry supported: latent_dim 512, rope_dim 64, scale groups of 64, page_tokens
 * a multiple of 128, q_len <= 2048.  cold tiles hold <= 128 tokens (int8: <= 64), hot/new tiles <= 32.
 */
typedef struct asterq_decode_params {
  int32_t n_heads;
  int32_t latent_dim;
  int32_t rope_dim;
  int32_t group_size;
  int32_t page_tokens;
  int32_t out_dtype; /* ASTERQ_DTYPE_F32 or ASTERQ_DTYPE_BF16 */
  float softmax_scale;
  float logit_softcap; /* <= 0: off */
  int64_t n_cold_pages;
  int64_t n_hot_pages;
  int64_t total_q;
  int32_t n_tiles;
  int32_t n_items;
  int32_t n_combine;
  int32_t n_slots;
  const void* q_lat;
  const void* q_rope;
  const void* new_latent;
  const void* new_rope;
  const void* cold_codes;
  const void* cold_scales;
  const void* cold_rope;
  const void* hot_latent;
  const void* hot_rope;
  const int32_t* tiles;
  const int32_t* items;
  const int32_t* combine;
  void* out;
  void* workspace;
  int64_t workspace_bytes;
  int32_t* device_status; /* optional int32 on the device: set nonzero if a pipeline wait timed out */
  const int32_t* units;   /* [n_units][2] {out_row0, n_rows}: the 16-row query blocks, prepared once per step */
  int32_t n_units;
  int32_t cold_scheme;    /* ASTERQ_SCHEME_HADAMARD_INT4 (0): cold codes rotated by the normalized Hadamard
                             transform (kv.py scheme "hadamard_int4"); ASTERQ_SCHEME_INT4: plain groupwise
                             int4 codes (scheme "int4"), same packing and scale layout */
  const int32_t* workers; /* optional [n_workers + 1] int32: CTA w runs items workers[w] .. workers[w + 1] - 1
                             in order (a balanced, persistent schedule); NULL: one CTA per item */
  int32_t n_workers;
  int32_t n_combine_total;  /* jobs in `combine`: [0, n_combine) run by the combine launch,
                               [n_combine, n_combine_total) by the decode kernel itself (unit_jobs) */
  const int32_t* unit_jobs; /* optional [n_units] int32: the combine job (index in [n_combine,
                               n_combine_total)) that the decode kernel runs itself, in the CTA that
                               writes the unit's last partial record, or -1.  NULL: none. */
  int64_t wait_limit_cycles; /* bound of every pipeline wait inside the kernel, in SM clock cycles;
                                0: the default (4e9, about 2 s).  A wait that runs out sets
                                *device_status (when given) and the kernel stops without hanging. */
  const int32_t* plan_counts; /* optional, device: the counts a device-built schedule wrote
                                 (asterq_plan_batch); the table sizes above are then its capacities:
                                 query blocks beyond counts[1] are not prepared, jobs [0, counts[6])
                                 run in the combine launch (n_combine is its grid), the others in
                                 the decode kernel.  NULL: the sizes above are exact. */
  int32_t rope_scheme;        /* ASTERQ_ROPE_BF16 (0) or ASTERQ_ROPE_QUANTIZED: the cold RoPE keys are
                                 INT4 codes of the cold scheme with one fp16 scale per token
                                 (LatentLayerCache quantize_rope=True, cache.py:160-164 -> kv.py:76-118);
                                 the kernel scores them on the int8 tensor path like a ninth latent
                                 group.  Hot and new tokens keep bf16 RoPE keys. */
  const void* cold_rope_scales; /* fp16 [n_cold_pages * page_tokens], 16-byte aligned (quantized RoPE keys
                                   of the INT4 schemes and int8; NULL for float8) */
} asterq_decode_params;

/*
 * Device-side schedule for a ragged, paged batch (continuous batching): the same tables the
 * host planner builds (tiles, units, items, workers, combine jobs), built on the GPU from page
 * tables and lengths that live on the GPU, so a decode loop that appends tokens to every
 * sequence each step replans without a host round trip (and can be recorded in a CUDA graph).
 * Replaces the host-side walk of the cache (cache.py:139-159 iter_chunks) by one small kernel.
 *
 * Sequence s: cold pages cold_pages[s][0 .. n_cold_pages[s]) oldest first, page j holding
 * cold_page_tokens[s][j] tokens from offset 0; a hot window of hot_tokens[s] tokens in pages
 * hot_pages[s][0 ..] (every page full except the last); q_len[s] new tokens at rows
 * q_start[s] .. of the step's arrays (q_len[s] <= 0: an empty slot, planned as nothing).
 * Tiles of a sequence: cold (<= cold_tile_tokens, never across a page), hot (<= 32), new (<= 32);
 * every 16-row query block is a unit; the units' tile ranges are cut into one contiguous share
 * per worker of equal estimated time.
 */
typedef struct asterq_batch_desc {
  int32_t n_seqs;
  int32_t n_heads;
  int32_t page_tokens;      /* a multiple of 16 */
  int32_t max_cold_pages;   /* row stride of cold_pages and cold_page_tokens */
  int32_t max_hot_pages;    /* row stride of hot_pages */
  int32_t n_workers;        /* worker CTAs (the decode grid), typically the SM count */
  const int32_t* n_cold_pages;      /* [n_seqs] */
  const int32_t* cold_pages;        /* [n_seqs][max_cold_pages] */
  const int32_t* cold_page_tokens;  /* [n_seqs][max_cold_pages] */
  const int32_t* hot_tokens;        /* [n_seqs] */
  const int32_t* hot_pages;         /* [n_seqs][max_hot_pages] */
  const int32_t* q_len;             /* [n_seqs], <= 2048 */
  const int32_t* q_start;           /* [n_seqs] */
  int32_t cold_tile_tokens;         /* tokens of a cold tile: 128 (0 means 128) for the INT4 schemes,
                                       64 for int8 codes (the decode kernel's cold tile of that scheme) */
} asterq_batch_desc;

/* Device tables asterq_plan_batch writes, sized by capacities chosen by the caller. */
typedef struct asterq_plan_buffers {
  int32_t cap_tiles;
  int32_t cap_units;
  int32_t cap_items;   /* also the partial-record slots; cap_units + n_workers always suffices */
  int32_t* tiles;      /* [cap_tiles][4] */
  int32_t* units;      /* [cap_units][2] */
  int32_t* items;      /* [cap_items][8] */
  int32_t* combine;    /* [cap_units][4]: jobs [0, counts[6]) for the combine launch, then the fused ones */
  int32_t* unit_jobs;  /* [cap_units] */
  int32_t* workers;    /* [n_workers + 1] */
  int32_t* counts;     /* [8]: n_tiles, n_units, n_items, n_slots, n_jobs, status (1: a capacity was
                          exceeded, nothing is planned), n_separate (jobs for the combine launch), 0 */
  void* scratch;       /* asterq_plan_scratch_bytes(...) bytes */
} asterq_plan_buffers;

/* Scratch bytes asterq_plan_batch needs for this descriptor's n_seqs, max_cold_pages and
 * n_workers and these capacities (0 on bad arguments). */
int64_t asterq_plan_scratch_bytes(const asterq_batch_desc* d, int32_t cap_tiles, int32_t cap_units,
                                  int32_t cap_items);

/* Enqueue the planner (one CTA).  Decode with the tables it wrote: asterq_latent_decode with
 * tiles/units/items/combine/unit_jobs/workers, n_tiles/n_units/n_items = the capacities,
 * n_slots = cap_items, n_combine = (n_workers + 15) / 16 (a unit goes to the combine launch
 * only when cut into more than 16 pieces, and every cut is a distinct worker boundary),
 * n_combine_total = cap_units, n_workers, plan_counts = counts. */
int asterq_plan_batch(const asterq_batch_desc* d, const asterq_plan_buffers* b, void* stream);

/* Append a step's new tokens to the hot windows in place (cache.py:195-200 without the
 * re-concatenation): for every s with q_len[s] > 0, rows q_start[s] .. q_start[s] + q_len[s] - 1
 * of new_latent (bf16 [total_q, 512]) and new_rope (bf16 [total_q, 64]) go to hot positions
 * hot_tokens[s] .. of the sequence's hot pages, then hot_tokens[s] += q_len[s].  `hot_tokens` is
 * the writable array (d->hot_tokens is not read).  A sequence whose positions reach a page that
 * is not in hot_pages (beyond max_hot_pages, or an id outside [0, n_hot_pool_pages)), or whose
 * rows pass total_q, is left unchanged and sets *status = 1 (status may be NULL).  One CTA per
 * sequence. */
int asterq_batch_append(const asterq_batch_desc* d, int32_t* hot_tokens, const void* new_latent,
                        const void* new_rope, int64_t total_q, void* hot_latent, void* hot_rope,
                        int64_t n_hot_pool_pages, int32_t* status, void* stream);

/* Bytes of workspace asterq_latent_decode needs: n_slots partial records of 32,896 B
 * (16 x 514 fp32), n_units prepared query blocks of 35,328 B, then one int32 counter per
 * unit (rounded up to 16 bytes) for the fused combine jobs. */
int64_t asterq_decode_workspace_bytes(const asterq_decode_params* p);

/* Enqueue the split-KV decode (and, when n_combine > 0, the combine). */
int asterq_latent_decode(const asterq_decode_params* p, void* stream);

/*
 * Same as asterq_latent_decode, but allocates nothing and ignores
 * p->workspace / p->workspace_bytes: the split-KV partial records and the
 * prepared query blocks go to a fixed array inside this library (room for 256
 * records and 256 query blocks, about 17.5 MB on every GPU that loads the
 * library, kept until the process exits).  No counterpart in
 * the reference; it exists for callers that cannot allocate device memory at
 * decode time (pre-planned serving loops, plain C hosts that only hold pointers
 * to their inputs and outputs).
 *   - Schedules needing more than 256 partial records or 256 query blocks
 *     (16 query rows each) are rejected with ASTERQ_ERR_WORKSPACE.
 *   - The first call on a device resolves the array's address; make that first
 *     call before any stream capture.
 *   - All calls share the one array: calls that overlap on the GPU (for
 *     example on two streams) race and corrupt each other's results.
 */
int asterq_latent_decode_noalloc(const asterq_decode_params* p, void* stream);

/*
 * Merge split-KV partial records with the online-softmax rule of
 * latent_attention.py:212-220 (used by the decode itself and by the
 * context-parallel path after the partials of all ranks are gathered).
 *   partials  float32: o [n_slots][16][latent_dim] (unnormalized), then m [n_slots][16], then l [n_slots][16]
 *   combine   int32   [n_combine][4] as in asterq_decode_params
 *   out       rows of latent_dim in out_dtype (float32 or bfloat16); job row r goes to row out_row0 + r
 */
int asterq_splitkv_combine(const float* partials, int32_t n_slots, const int32_t* combine, int32_t n_combine,
                           int32_t latent_dim, void* out, int32_t out_dtype, void* stream);

/*
 * Merge split-KV partial records into fewer partial records with the same rule,
 * without normalising: job j (combine table layout; out_row0 / n_rows unused)
 * turns slots [slot_begin, slot_end) into record j of `merged`, which has the
 * workspace layout (o [n_jobs][16][latent_dim], m [n_jobs][16], l [n_jobs][16]).
 * Used by context-parallel decode before the ranks' records are gathered;
 * replaces the per-chunk merge step of latent_attention.py:212-220 applied
 * across ranks.
 */
int asterq_splitkv_merge(const float* partials, int32_t n_slots, const int32_t* jobs, int32_t n_jobs,
                         int32_t latent_dim, float* merged, void* stream);

/*
 * Combine the merged records of `world` ranks as a rank-major all-gather leaves
 * them: rank r's part, at gathered + r * n_blocks * 16 * (latent_dim + 2), is the
 * asterq_splitkv_merge output for n_blocks jobs (o [n_blocks][16][latent_dim],
 * m [n_blocks][16], l [n_blocks][16]).  jobs int32 [n_blocks][4]: job b merges
 * record b of ranks [slot_begin, slot_end) (normally 0 and world) into rows
 * out_row0 .. out_row0 + n_rows - 1 of `out`.  Same rule as
 * asterq_splitkv_combine (latent_attention.py:212-220 applied across ranks),
 * with no reordering copy of the gathered records first.
 */
int asterq_splitkv_combine_ranks(const float* gathered, int32_t world, int32_t n_blocks, const int32_t* jobs,
                                 int32_t latent_dim, void* out, int32_t out_dtype, void* stream);

/*
 * Context-parallel record exchange by peer stores, in place of the all-gather above (the
 * reference has no multi-GPU code; this replaces the collective that
 * asterq_splitkv_merge + all_gather + asterq_splitkv_combine_ranks need, with the same
 * merge rule, latent_attention.py:212-220, across ranks).
 *
 * Every rank creates one mailbox (device memory of asterq_mailbox_bytes bytes, zeroed) and
 * gets a CUDA IPC handle for it; the ranks exchange handles on the host, and each maps its
 * peers' mailboxes with asterq_mailbox_open.  A step on each rank, on one stream:
 *   asterq_latent_decode  (split-KV partial records in the workspace, n_combine = 0)
 *   asterq_cp_merge_push  merges them into one record per 16-row block (jobs as for
 *                         asterq_splitkv_merge) and stores it into slot `rank` of every rank's
 *                         mailbox (mailboxes: a device array of `world` pointers, this rank's
 *                         own mailbox at index `rank`, the mapped peers' at theirs), then raises
 *                         this rank's flag in every mailbox to the step number;
 *   asterq_cp_combine_wait waits until every rank's flag in this rank's mailbox has reached the
 *                         step (bounded by wait_limit_cycles SM cycles, 0: about 2 s; on timeout
 *                         *status = 1 and `out` is left unwritten), then combines all ranks'
 *                         records as asterq_splitkv_combine_ranks does (jobs likewise).
 * Steps alternate between two record buffers; every rank must run the same steps.  No TMA or
 * library kernel reads a peer's memory: records cross NVLink as plain stores.  Close the peer
 * mappings and destroy the mailboxes only after every rank has finished its last step.
 * world <= 56.
 */
#define ASTERQ_IPC_HANDLE_BYTES 64
int64_t asterq_mailbox_bytes(int32_t world, int32_t n_blocks, int32_t latent_dim);
int asterq_mailbox_create(int64_t bytes, void** dev_ptr, void* ipc_handle /* ASTERQ_IPC_HANDLE_BYTES out */);
int asterq_mailbox_open(const void* ipc_handle, void** peer_ptr);
int asterq_mailbox_close(void* peer_ptr);
int asterq_mailbox_destroy(void* dev_ptr);
int asterq_cp_merge_push(const float* partials, int32_t n_slots, const int32_t* jobs, int32_t n_blocks,
                         int32_t latent_dim, void* const* mailboxes, int32_t world, int32_t rank, void* stream);
int asterq_cp_combine_wait(const void* mailbox, int32_t world, int32_t n_blocks, const int32_t* jobs,
                           int32_t latent_dim, void* out, int32_t out_dtype, int64_t wait_limit_cycles,
                           int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ASTERQ_H_ */
