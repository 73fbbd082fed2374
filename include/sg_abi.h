/*
 * sg_abi.h -- C-ABI of the B200 SlottedGLU MoE hot path (libsg_b200.so).
 *
 * Every entry point is extern "C", takes plain device pointers, sizes and a
 * cudaStream_t passed as void*, returns an int status (SG_OK == 0, negative on
 * error) and never throws.  The caller owns every buffer.  No entry point
 * synchronises the stream except sg_refill_h2d's optional host wait.
 *
 * bf16 values are passed as uint16_t bit patterns.  A call whose token or pair
 * count is 0 returns SG_OK without touching its (possibly NULL) data pointers.  Layout conventions follow
 * the reference (preemptLM, preempt/backends/mlx_metal/...):
 *   x        [T, H]            bf16 hidden states, row-major
 *   router   [E, H]            bf16 (mlx_lm nn.Linear weight, out x in)
 *   arena    gate/up [S, I, H], down [S, H, I]   (SlottedGLU, expert_cache.py:199-224)
 *            or MLX affine: packed uint32 [S, out, in*bits/32] little-endian,
 *            scales/biases bf16 [S, out, in/group_size]
 *   pairs    p = t*k + j  (token t, routing rank j)
 */
#ifndef SG_ABI_H
#define SG_ABI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
enum sg_status {
  SG_OK = 0,
  SG_ERR_INVALID_ARG = -1,   /* null pointer / negative size */
  SG_ERR_SHAPE = -2,         /* unsupported dimension (see each call) */
  SG_ERR_FORMAT = -3,        /* unsupported weight format (bits / group size) */
  SG_ERR_CUDA = -4,          /* a CUDA runtime call or launch failed */
  SG_ERR_CAPACITY = -5,      /* a caller buffer is too small */
  SG_ERR_TIMEOUT = -6,       /* a bounded wait gave up */
};

/* Row order flags of sg_glu_gate_up / sg_glu_down.  Pair order: row p of the
 * pair index p = t * k + j (h, y; x is indexed by p / pair_div).  Dispatch
 * order: row pos of the sg_dispatch permutation (pairs grouped by expert). */
enum sg_glu_flags {
  SG_IN_DISPATCH_ORDER = 1,   /* input rows are in dispatch order (num_pairs rows) */
  SG_OUT_DISPATCH_ORDER = 2,  /* write output rows in dispatch order */
};

/* Human-readable text of a status code (static storage). */
const char* sg_status_string(int status);

/* Library version, and the SM architecture the kernels were built for (1000). */
int sg_version(void);
int sg_built_arch(void);

/* --------------------------------------------------------------- the arena
 * Pre-allocated per-layer slot arena: SlottedGLU (expert_cache.py:199-224),
 * plus MLX affine 4/8-bit layouts (ops/fused.py:77-88 calling convention,
 * quantization.py:16-40 QuantSettings).  bits == 16 means plain bf16 weights
 * (scale/bias pointers unused).  group_size must be 64 for bits 4 and 8. */
typedef struct sg_arena {
  int32_t num_slots;  /* S */
  int32_t hidden;     /* H */
  int32_t inter;      /* I */
  int32_t bits;       /* 16, 8 or 4 */
  int32_t group_size; /* 64 (affine) */
  int32_t reserved;
  const void* gate_w; const void* gate_s; const void* gate_b;
  const void* up_w;   const void* up_s;   const void* up_b;
  const void* down_w; const void* down_s; const void* down_b;
} sg_arena;

/* ----------------------------------------------------------- router (a1)
 * logits[T, E] = bf16(x[T, H] @ w[E, H]^T), fp32 accumulation in a fixed order
 * (32 lane partials over h = 256*i + 8*lane + e, then a pairwise fold).
 * Replaces the router call `logits = self.inner.gate(x)` at
 * preempt/backends/mlx_metal/module_wrappers/qwen3_x_moe.py:254 and the shared
 * expert gate `self.inner.shared_expert_gate(x)` at qwen3_x_moe.py:259.
 * Requires H % 256 == 0, E >= 1. */
int sg_router_logits(const uint16_t* x, const uint16_t* w, uint16_t* logits,
                     int T, int H, int E, void* stream);

/* ---------------------------------------------------------- routing (a2)
 * softmax(precise) -> top-k in the order (gate desc, expert id asc) ->
 * optional renormalisation.  inds[T, k] int32, scores[T, k] bf16.
 * Replaces `_get_routings` at qwen3_x_moe.py:26-40.
 * Requires E % 32 == 0, E <= 1024, 1 <= k <= 32, k <= E. */
int sg_route_topk(const uint16_t* logits, int T, int E, int k, int norm_topk_prob,
                  int32_t* inds, uint16_t* scores, void* stream);

/* --------------------------------------------------------- dispatch (a3/a6)
 * Device-side replacement for the host part of `_maybe_admit`
 * (qwen3_x_moe.py:145-156: np.unique with inverse, the miss set) and for
 * `slot_ids = self._eid_lookup_table[unique_eids]` (qwen3_x_moe.py:277).
 * One CTA; all scratch lives in shared memory.
 *   in : inds[P] (P = T*k pair expert ids), eid2sid[E] (-1 = not resident)
 *   out: unique[U] ascending, inverse[P], counts[0] = U, counts[1] = #missed,
 *        slot_ids[U] = eid2sid[unique], miss_eids[#missed] ascending,
 *        group_off[U+1] (pairs of unique u are perm[group_off[u]..group_off[u+1]) ),
 *        perm[P] pair ids grouped by unique index.
 *   max_unique bounds unique/slot_ids/miss_eids/group_off (needs >= min(P, E) + 1).
 *   With P == 0, inds/inverse/perm may be NULL (counts and group_off[0] are still written).
 * Requires 1 <= E <= 8192. */
int sg_dispatch(const int32_t* inds, int P, int E, const int32_t* eid2sid,
                int32_t* unique, int32_t* inverse, int32_t* counts,
                int32_t* slot_ids, int32_t* miss_eids, int32_t* group_off,
                int32_t* perm, int max_unique, void* stream);

/* ------------------------------------------- fused routing + dispatch (a2/a3/a6)
 * sg_route_topk followed by sg_dispatch in one launch: softmax, top-k in the
 * order (gate desc, expert id asc) and renormalisation per token (one warp
 * per token), then the unique experts, inverse map, slot lookup, miss list,
 * group offsets and pair permutation, all with the outputs and meaning of
 * those two calls (inds/scores [T, k]; the sg_dispatch arrays for the
 * P = T * k pairs; the order of pairs inside a group is not specified).
 * work: caller-provided int32 [E + 1], all zero before the first call; every
 * call leaves it zero (calls using one work buffer must not overlap).
 * trace (NULL: none): the kernel also writes each token's ids, scores and
 * raw logits there as it produces them -- the router-selection telemetry that
 * the reference's recorder captures, `self.recorder.capture(...)` at
 * qwen3_x_moe.py:261-269 (recorder.py:57-111), without another launch.
 * Replaces `_get_routings` (qwen3_x_moe.py:26-40), the host np.unique and
 * miss set of `_maybe_admit` (:145-156) and `slot_ids =
 * self._eid_lookup_table[unique_eids]` (:277).
 * Requires E % 32 == 0, E <= 1024, 1 <= k <= 32, k <= E; max_unique >=
 * min(P, E) + 1. */
typedef struct sg_route_trace {
  int32_t* ids;      /* [T, k] the routed expert ids, or NULL */
  uint16_t* scores;  /* [T, k] bf16 scores after renormalisation, or NULL */
  uint16_t* logits;  /* [T, E] bf16 router logits (pre-softmax), or NULL */
} sg_route_trace;

int sg_route_dispatch(const uint16_t* logits, int T, int E, int k, int norm_topk_prob,
                      const int32_t* eid2sid, int32_t* inds, uint16_t* scores,
                      int32_t* unique, int32_t* inverse, int32_t* counts, int32_t* slot_ids,
                      int32_t* miss_eids, int32_t* group_off, int32_t* perm, int max_unique,
                      int32_t* work, const sg_route_trace* trace, void* stream);

/* Device address of pinned host memory (cudaHostGetDevicePointer), for
 * trace arrays the kernels write straight into host memory. */
int sg_host_device_ptr(void* host, void** device);

/* ------------------------------------------------- gathered SwiGLU (a9/a10)
 * y[p, H] = bf16(swiglu(x[p / pair_div] @ gate^T, ... @ up^T) @ down^T) for
 * every pair p of every group u < counts[0], against arena slot slot_ids[u];
 * pairs listed by perm/group_off (sg_dispatch layout); num_pairs = P (length
 * of perm, rows of y; x has ceil(P / pair_div) rows); y in pair order.
 * scratch and h [P, I] are caller-provided intermediate storage.  scratch
 * holds sg_glu_forward_scratch_bytes() bytes: the pairs' token rows copied
 * into dispatch order for prefill-sized groups (every tile's rows then load
 * as one TMA box), or, for the integer-operand kernels of 8-bit arenas at
 * decode sizes, the token rows' 8-bit pieces and afterwards h's (see
 * sg_quantize_pieces).  NULL is allowed when that size is 0, and also when
 * only pieces would go there (the dequantising kernels then run instead).
 * h is kept in dispatch order.
 * pair_div = k for routed experts.  grid_groups is a host-side upper bound
 * on counts[0].
 * Replaces `_gather_forward`, qwen3_x_moe.py:210-248 (the `mx.take` of the
 * arena, two `gather_mm` + `swiglu_activation`, the down `gather_mm`). */
int sg_glu_forward(const sg_arena* arena, const uint16_t* x, int num_pairs, int pair_div,
                   const int32_t* counts, const int32_t* slot_ids,
                   const int32_t* group_off, const int32_t* perm,
                   int grid_groups, void* scratch, uint16_t* h, uint16_t* y, void* stream);

/* Bytes of the scratch area sg_glu_forward uses for this problem (0: none),
 * or a negative status for invalid arguments.  Same arguments as
 * sg_glu_forward.  No counterpart in the reference. */
long long sg_glu_forward_scratch_bytes(const sg_arena* arena, int num_pairs, int pair_div, int grid_groups);

/* sg_glu_forward without caller scratch: h (and the permuted token rows when
 * sg_glu_use_permute returns 1) live in a fixed 32 MiB device-resident scratch
 * area of the library (a file-scope __device__ array, its address looked up
 * once per device), so the call allocates nothing.  Returns SG_ERR_CAPACITY
 * when num_pairs * inter * 2 bytes (rounded up to 256), plus num_pairs *
 * hidden * 2 when permuting, exceed 32 MiB.  Nothing in the scratch area needs
 * to start at zero.  Calls that overlap in time on one device (different
 * streams or host threads) share the area and race; calls on one stream are
 * ordered.  No counterpart in the reference. */
int sg_glu_forward_noalloc(const sg_arena* arena, const uint16_t* x, int num_pairs, int pair_div,
                           const int32_t* counts, const int32_t* slot_ids,
                           const int32_t* group_off, const int32_t* perm,
                           int grid_groups, uint16_t* y, void* stream);

/* 1 when sg_glu_forward permutes the token rows for this problem size. */
int sg_glu_use_permute(const sg_arena* arena, int num_pairs, int grid_groups);

/* xs[pos, :] = x[perm[pos] / pair_div, :] for pos < num_pairs (H % 8 == 0);
 * every perm[pos] must be written (a dispatch of ids without -1 entries).
 * sg_glu_forward permutes only the filled positions itself. */
int sg_permute_rows(const uint16_t* x, const int32_t* perm, int pair_div, int num_pairs, int H,
                    uint16_t* xs, void* stream);

/* sg_permute_rows over the filled pair positions of a dispatch only (pos <
 * group_off[counts[0]]), so ids of -1 (padded expert-parallel inboxes) are
 * allowed; rows past the filled ones are left as they are. */
int sg_permute_pairs(const uint16_t* x, const int32_t* perm, int pair_div, const int32_t* counts,
                     const int32_t* group_off, int num_pairs, int H, uint16_t* xs, void* stream);

/* The two halves of sg_glu_forward.  h[., I] = swiglu(x @ gate^T, x @ up^T)
 * per pair; rows in pair or dispatch order per `flags` (sg_glu_flags; input
 * in dispatch order means x has num_pairs rows and pair_div is not used).
 * Rounds x_up, x_gate, sigmoid, silu and the product to bf16
 * (experts.py:26-28).  Replaces the up/gate `gather_mm` calls and
 * `swiglu_activation` in `_gather_forward`, qwen3_x_moe.py:225-242.
 * Requires H % 64 == 0 and I % 64 == 0. */
int sg_glu_gate_up(const sg_arena* arena, const uint16_t* x, int num_pairs, int pair_div,
                   const int32_t* counts, const int32_t* slot_ids,
                   const int32_t* group_off, const int32_t* perm,
                   int grid_groups, uint16_t* h, int flags, void* stream);

/* sg_glu_gate_up with a caller work area of work_bytes bytes: with 8-bit
 * arenas at decode tile widths, and work_bytes >= sg_glu_gate_up_work_bytes(),
 * the token rows are split into 8-bit pieces in the work area and the
 * integer-operand tcgen05 kernel computes h (never dequantising the
 * weights: sum_g scale * (q . x)_g + bias * (sum x)_g per 64-group); any
 * other case runs sg_glu_gate_up's kernels.  h agrees with the dequantising
 * kernels within the layer tolerance (the pieces hold every token element
 * to 2^-14 of its group's largest magnitude; the weights are exact).
 * Same replacement as sg_glu_gate_up. */
long long sg_glu_gate_up_work_bytes(const sg_arena* arena, int num_pairs, int pair_div, int grid_groups,
                                    int flags);
int sg_glu_gate_up_work(const sg_arena* arena, const uint16_t* x, int num_pairs, int pair_div,
                        const int32_t* counts, const int32_t* slot_ids,
                        const int32_t* group_off, const int32_t* perm,
                        int grid_groups, uint16_t* h, int flags, void* work, long long work_bytes,
                        void* stream);

/* 8-bit pieces of rows x K bf16 values (K % 64 == 0), per 64-group g of a
 * row: x[k] = E * (256 * hi[k] + lo[k]) with E = 2^e the group's scale,
 * chosen so the largest |x| of the group is below 2^14 * E; hi in [-64, 64],
 * lo in [-128, 127]; an element's integer is exact when it lies within 2^6
 * of the group's largest magnitude, else rounded to nearest.  pieces
 * [rows, 2, K] int8 (hi row, then lo row); ex [rows, K / 64, 2] fp32 (E, E *
 * sum(256 hi + lo)).  order 1 stores every 8 elements in the order
 * 0,2,4,6,1,3,5,7.  Finite inputs only.  No counterpart in the reference. */
int sg_quantize_pieces(const uint16_t* x, int rows, int K, int order, int8_t* pieces, float* ex,
                       void* stream);

/* y[., H] = bf16(h[., I] @ down^T) for every listed pair (num_pairs rows),
 * orders per `flags`.  Replaces the down `gather_mm` in `_gather_forward`,
 * qwen3_x_moe.py:243-248. */
int sg_glu_down(const sg_arena* arena, const uint16_t* h, int num_pairs,
                const int32_t* counts, const int32_t* slot_ids,
                const int32_t* group_off, const int32_t* perm,
                int grid_groups, uint16_t* y, int flags, void* stream);

/* sg_glu_down with a caller work area: with 8-bit arenas at decode tile
 * widths and work_bytes >= sg_glu_down_work_bytes(), h is split into 8-bit
 * pieces in the work area and the integer-operand tcgen05 kernel computes y
 * (256-row tiles); otherwise sg_glu_down's kernels run.  Same replacement as
 * sg_glu_down. */
long long sg_glu_down_work_bytes(const sg_arena* arena, int num_pairs, int grid_groups);
int sg_glu_down_work(const sg_arena* arena, const uint16_t* h, int num_pairs,
                     const int32_t* counts, const int32_t* slot_ids,
                     const int32_t* group_off, const int32_t* perm,
                     int grid_groups, uint16_t* y, int flags, void* work, long long work_bytes,
                     void* stream);

/* Dense SwiGLU of one slot over every row: h[t, I] = swiglu(x @ gate^T, x @ up^T),
 * y[t, H] = bf16(h @ down^T) for t < T, slot sid of the arena (the shared
 * expert: one slot, all tokens).  h is caller-provided intermediate storage.
 * Replaces `self.inner.shared_expert(x)`, qwen3_x_moe.py:258.  Needs the
 * tensor-core shapes (H and I multiples of 128, packed rows of >= 128 bytes);
 * returns SG_ERR_SHAPE otherwise (sg_glu_gate_up / sg_glu_down over a
 * one-group dispatch serve those shapes). */
int sg_dense_glu(const sg_arena* arena, int sid, const uint16_t* x, int T, uint16_t* h, uint16_t* y,
                 void* stream);

/* Kernel choice for sg_glu_forward / sg_glu_gate_up / sg_glu_down: 0 =
 * automatic: tcgen05 when the shape allows (in-dim % 64, out-dim % 128,
 * <= 2048 groups) and either the mean pairs per group is >= 4 or the groups
 * make at least one weight tile per SM (128 rows for gate/up, 256 for down),
 * else the streaming GEMV; on tcgen05, the integer-operand kernels for 8- and
 * 4-bit arenas while the mean is <= 16 and the caller passes a work area, the
 * token rows permuted once the mean reaches 32.  1 = streaming GEMV always,
 * 2 = the dequantising tcgen05 kernels whenever the shape allows, 3 = as 2
 * with the token rows always permuted, 4 = tcgen05 whenever the shape allows,
 * with the integer-operand kernels wherever they apply.  Process-wide.  No
 * counterpart in the reference (MLX picks its own gather_mm kernels). */
int sg_set_glu_path(int mode);

/* Pair-tile width: 0 = automatic (integer-operand kernels 8 while groups
 * average at most 6 pairs, else 16; dequantising kernels the smallest of
 * 16/32/64/128 that holds the mean group).  8 fixes the integer-operand
 * kernels' tile, 32, 64 or 128 the dequantising kernels', 16 both.
 * Process-wide.  No counterpart in the reference. */
int sg_set_glu_tile(int bn);

/* First error a kernel of this library recorded on the current device since
 * the last reset (SG_OK if none; SG_ERR_TIMEOUT when a bounded wait inside a
 * kernel expired and the kernel gave up).  Synchronises with the device.
 * No counterpart in the reference (MLX raises host exceptions). */
int sg_device_status(int reset);

/* ---------------------------------------------------------- combine (a11)
 * out[t] = bf16( bf16(sum_j bf16(y[t*k+j] * scores[t, j]))
 *               + bf16(bf16(sigmoid(shared_gate[t])) * shared_y[t]) )
 * The k-sum adds in fp32 in j order.  shared_y / shared_gate may both be NULL
 * (no shared expert).  Replaces `_combine_shared`, qwen3_x_moe.py:71-80.
 * Requires H % 8 == 0. */
int sg_combine(const uint16_t* y, const uint16_t* scores, int T, int k, int H,
               const uint16_t* shared_y, const uint16_t* shared_gate,
               uint16_t* out, void* stream);

/* ------------------------------------------------------------ refill (a8)
 * Copies one serialized expert blob (pinned host memory, tensors concatenated
 * in the bank's tensor_specs order: gate, up, down x weight[, scales, biases])
 * into arena slot `sid` with one cudaMemcpyAsync per tensor on `stream`.
 * Replaces `decode_serialized_expert` + the slot writes
 * `self._weight_slots.{up,down,gate}_proj[sid] = ...` at
 * qwen3_x_moe.py:186-195 (expert_cache.py:24-80).  blob_len must equal the
 * expert's byte size for the arena format, else SG_ERR_SHAPE. */
int sg_refill_h2d(const void* blob, size_t blob_len, const sg_arena* arena,
                  int sid, void* stream);

/* Byte size of one expert blob in the arena's format. */
size_t sg_expert_bytes(const sg_arena* arena);

/* ------------------------------------------ expert-parallel exchange (e)
 * The dispatch / combine all-to-alls of one expert-parallel layer over
 * NVLink peer memory, one process per GPU, R <= 8 ranks in lockstep.  No
 * counterpart in the reference (it runs on one device); these replace the
 * NCCL counts / rows / outputs all-to-alls of the expert-parallel layer.
 *
 * Each rank allocates one region (sg_ep_alloc, sg_ep_region_bytes(R, cap, H)
 * bytes, zeroed), exports it with sg_ep_ipc_handle, and opens every peer's
 * with sg_ep_ipc_open; `regions` lists all R regions in this process's
 * address space (its own included), in rank order.  cap = the most tokens
 * per rank per step times k.  Every rank runs the same number of steps; the
 * step number lives in the region (sg_ep_send bumps it), so a step captured
 * in a CUDA graph replays correctly.  Per step:
 *   sg_ep_send(regions, R, me, cap, H, x [T, H], inds [T, k] global expert
 *     ids, T, k, per = experts per rank, dcnt [R] int32 counters, zero
 *     before the first call and left zero by every call): every pair's token
 *     row, local expert id and pair id into its owner's inbox, then that
 *     rank's step flag (T * k <= cap);
 *   sg_ep_wait_inbox(own region, ...): waits for every source's flag
 *     and marks unused inbox entries empty (expert id -1);
 *   sg_dispatch + sg_glu_gate_up / sg_glu_down then run over the R * cap
 *     inbox rows and ids (sg_ep_layout gives their offsets) in place;
 *   sg_ep_send_back(regions, ..., y [R * cap, H]): each filled entry's
 *     output row to its source, at its pair id, then the step flag;
 *   sg_ep_wait_back(own region, ..., inds, T, k, per): waits for every
 *     owner's flag; the region's pair-order output rows ([T * k, H], offset 4
 *     of sg_ep_layout) are then complete for sg_combine.
 * Every wait is bounded (2 s by default, sg_ep_set_wait_limit); on expiry
 * sg_device_status reports SG_ERR_TIMEOUT, sg_ep_wait_inbox marks the late
 * source's inbox empty and sg_ep_wait_back zeroes the output rows of the
 * pairs owned by the late rank.  A timed-out exchange is out of step (a late
 * peer may still write into the region): free it and build a new one.
 * Calls of one exchange must be issued on one stream, one step at a time
 * (the finished-CTA counters of a rank's send kernels live in its region).
 * Allocation, IPC and freeing are set-up calls (they synchronise); free a
 * region only after every rank has stopped using it. */
long long sg_ep_region_bytes(int R, int cap, int H);
/* offsets5: byte offsets of rows [R*cap][H] bf16, eids [R*cap] int32,
 * pair ids [R*cap] int32, counts [R] int32, outputs [cap][H] bf16. */
int sg_ep_layout(int R, int cap, int H, long long* offsets5);
int sg_ep_alloc(long long bytes, void** region);
int sg_ep_free(void* region);
int sg_ep_ipc_handle(void* region, uint8_t* handle64);
int sg_ep_ipc_open(const uint8_t* handle64, void** region);
int sg_ep_ipc_close(void* region);
int sg_ep_send(void* const* regions, int R, int me, int cap, int H, const uint16_t* x, const int32_t* inds,
               int T, int k, int per, int32_t* dcnt, void* stream);
int sg_ep_wait_inbox(void* region, int R, int cap, int H, void* stream);
int sg_ep_send_back(void* const* regions, int R, int me, int cap, int H, const uint16_t* y, void* stream);
int sg_ep_wait_back(void* region, int R, int cap, int H, const int32_t* inds, int T, int k, int per,
                    void* stream);
/* Wait limit of the exchange kernels launched after this call on the current
 * device, in microseconds (1 .. 600e6; default 2e6).  Synchronous. */
int sg_ep_set_wait_limit(long long microseconds);

#ifdef __cplusplus
}
#endif

#endif /* SG_ABI_H */
