/*
 * moe_b200.h -- C ABI of libmoe_b200.so, the B200 (sm_100a) MoE layer behind
 * lightreason's edge35b expert-forward operator API.
 *
 * Conventions (all entry points):
 *   - plain pointers and sizes; BF16 values travel as uint16_t bit patterns;
 *   - every pointer to tensor data is a device pointer (or a CUDA-mapped pinned
 *     host pointer where an entry point says so);
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *     work is enqueued on it and the call returns without synchronising;
 *   - the return value is a status: MOE_OK, or MOE_EINVAL for argument errors
 *     (the Python layer raises ValueError, as the reference does for shape and
 *     dtype violations: edge35b/fused_experts.py:41-50), MOE_ECUDA for a CUDA
 *     failure (RuntimeError, as edge35b/native_bf16_gather.py:25-29 _checked),
 *     MOE_EARCH when the device is not sm_100; moe_last_error() describes the
 *     last failure on the calling thread;
 *   - an empty batch (tokens == 0) is a no-op for the router, permute, layer,
 *     combine and shared-expert entry points, as it is for the eager module:
 *     their per-token arrays may then be NULL (shapes are still checked; the
 *     permute still writes zero offsets and num_active); the expert-parallel
 *     step needs at least one token per rank;
 *   - no entry point allocates device memory unless its comment says so.
 *     Scratch lives in a caller-owned workspace sized by a *_workspace_bytes
 *     query; entry points that read routing counts do so on the device, so a
 *     call can be captured in a CUDA graph and replayed with new routes.
 */
#ifndef LIGHTREASON_B200_MOE_H
#define LIGHTREASON_B200_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_OK 0
#define MOE_EINVAL 1
#define MOE_ECUDA 2
#define MOE_EARCH 3

/* Library version (major*10000 + minor*100 + patch). */
int moe_version(void);

/* Description of the last nonzero status returned on this thread. */
const char *moe_last_error(void);

/* MOE_OK when `device` is an sm_100 GPU this build can run on. */
int moe_device_check(int device);

/* Page-lock and map a host range for zero-copy device reads (the pinned host
 * expert banks read by moe_gather_*).  Replaces the pinned staging set-up of
 * edge35b/expert_stream.py:177-198 (_PackedBuffers) and FreeToken's
 * device_ptr() mapping (edge35b/gpu_resident_experts.py:159,228).  Returns the
 * device address of `ptr` in *device_ptr. */
int moe_host_register(void *ptr, size_t bytes, uint64_t *device_ptr);
int moe_host_unregister(void *ptr);

/* ------------------------------------------------------------------------
 * Router.  Replaces Qwen3_5MoeTopKRouter.forward (transformers
 * models/qwen3_5_moe/modeling_qwen3_5_moe.py:762-770, the third-party router
 * edge35b calls) and the shared_expert_gate Linear (same file :779, :788).
 *
 * logits[t][e] = bf16(x[t] . router[e]) (FP32 accumulation), then per token
 * z = float(logits) + bias (bias may be NULL), softmax(z), top_k by z with
 * exact ties to the lower expert id, weights w_k = p_k / sum_k p_k written as
 * FP32 (scores_f32, may be NULL) and BF16 (scores_bf16, may be NULL).
 * If shared_gate_w != NULL, sig[t] = bf16(sigmoid(bf16(x[t] . shared_gate_w))).
 * x [T,H] row-major; router [E,H]; idx [T,top_k] int64; logits [T,E] is a
 * required output (it is also the scratch between the two halves).
 * hidden in {1024,2048,4096}, experts <= 1024, top_k <= 32.
 * ------------------------------------------------------------------------ */
int moe_router_topk(const uint16_t *x, const uint16_t *router, const float *bias,
                    const uint16_t *shared_gate_w, int tokens, int hidden, int experts,
                    int top_k, uint16_t *logits, int64_t *idx, float *scores_f32,
                    uint16_t *scores_bf16, uint16_t *sig, void *stream);

/* moe_router_topk with a scratch for FP32 K-split partials of the router GEMM
 * at prefill widths (more CTAs when few tokens), summed in split order before
 * the one BF16 rounding: the router moe_layer_forward runs, bit for bit.
 * moe_router_topk itself accumulates K in one pass, so where this call splits
 * a logit may differ from it by the rounding of the FP32 sum.
 * moe_router_workspace_bytes: the scratch it uses (0: none, and the call is
 * moe_router_topk). */
size_t moe_router_workspace_bytes(int tokens, int experts);
int moe_router_topk_ws(const uint16_t *x, const uint16_t *router, const float *bias,
                       const uint16_t *shared_gate_w, int tokens, int hidden, int experts,
                       int top_k, uint16_t *logits, int64_t *idx, float *scores_f32,
                       uint16_t *scores_bf16, uint16_t *sig, void *workspace,
                       size_t workspace_bytes, void *stream);

/* Selection only, from given BF16 logits [T,E] (the router's second half). */
int moe_router_select(const uint16_t *logits, const float *bias, int tokens, int experts,
                      int top_k, int64_t *idx, float *scores_f32, uint16_t *scores_bf16,
                      void *stream);

/* ------------------------------------------------------------------------
 * Token permute.  Replaces the eager dispatch order of
 * Qwen3_5MoeExperts.forward (modeling_qwen3_5_moe.py:730-744: ascending
 * expert, then slot-major, then token) and edge35b/pipeline.py:59-76 _routes.
 * Outputs: offsets[E+1] (exclusive scan of per-expert counts), perm_token[R],
 * perm_slot[R] (route position -> token, slot), route_pos[T*top_k] ((token,
 * slot) -> position), active[E] (experts with routes, ascending) and
 * num_active[1].  R = tokens*top_k.  Ids outside [0,E) are dropped and counted
 * in *bad_routes (may be NULL).  Requires experts <= 1024.
 * ------------------------------------------------------------------------ */
int moe_permute(const int64_t *idx, int tokens, int top_k, int experts, int32_t *offsets,
                int32_t *perm_token, int32_t *perm_slot, int32_t *route_pos, int32_t *active,
                int32_t *num_active, int32_t *bad_routes, void *stream);

/* The same permute, same outputs, for many routes: above 2048 routes it runs
 * on many CTAs (per-chunk counts, a column scan, placement) with a caller scratch
 * `hist` of moe_permute_hist_ints(tokens, top_k, experts) int32s (0: not
 * needed, and moe_permute runs). */
int moe_permute_hist_ints(int tokens, int top_k, int experts);
int moe_permute_wide(const int64_t *idx, int tokens, int top_k, int experts, int32_t *offsets,
                     int32_t *perm_token, int32_t *perm_slot, int32_t *route_pos, int32_t *active,
                     int32_t *num_active, int32_t *bad_routes, int32_t *hist, void *stream);

/* ------------------------------------------------------------------------
 * Expert rows by pointer table, the GPU counterpart of edge35b/cpu_experts.c.
 *
 * moe_expert_rows replaces expert_rows (cpu_experts.c:43-71, bound by
 * edge35b/cpu_route.py:10-20): output[e] = the BF16 down projection of the one
 * token `input` [H] through expert e, for e < experts (<= 128), with
 * gate_up[e] -> [2I,H] and down[e] -> [H,I] device pointers (host arrays of
 * device pointers).  H = 2048, I = 512 as in cpu_experts.c:7-9.
 *
 * moe_expert_block_rows replaces expert_block_rows (cpu_experts.c:74-105,
 * bound by edge35b/block_experts.py:52-59): pair e reads token token_ids[e] of
 * input [tokens,H]; tokens <= 16, experts <= 128 as in cpu_experts.c:77-78.
 *
 * gate_up, down and token_ids are HOST arrays (as the reference's ctypes
 * arrays); input, output and the weights they point to are device memory.
 * The reference keeps the [experts, 512] intermediate activations on its
 * stack; on the GPU they live in a caller workspace of >= experts*512*2 bytes.
 * ------------------------------------------------------------------------ */
int moe_expert_rows(const uint16_t *const *gate_up, const uint16_t *const *down,
                    const uint16_t *input, uint16_t *output, int experts, void *workspace,
                    size_t workspace_bytes, void *stream);
int moe_expert_block_rows(const uint16_t *const *gate_up, const uint16_t *const *down,
                          const uint16_t *input, const int32_t *token_ids, uint16_t *output,
                          int tokens, int experts, void *workspace, size_t workspace_bytes,
                          void *stream);

/* Allocation-free variant of moe_expert_block_rows.  It has no counterpart in
 * the reference.  It serves callers that hold only device pointers and cannot
 * allocate device memory (a C/C++ worker in the place of the reference's
 * cpu_experts.c call, or a server that forbids allocation once it runs): the
 * [experts, 512] activations live in a 128 KiB array inside the library
 * instead of a caller workspace.  At most 128 pairs (larger tables are
 * rejected with MOE_EINVAL); token_ids == NULL means one token (expert_rows).
 * The first call on each device looks up the array's device address; make it
 * before any stream capture.  The address is kept for the life of the
 * process: do not call this entry point again on a device after
 * cudaDeviceReset (or any reset of its primary context), which would leave
 * the kept address stale.  All calls on a device share the array: calls
 * that can overlap on the GPU race and must be ordered on one stream. */
int moe_expert_block_rows_noalloc(const uint16_t *const *gate_up, const uint16_t *const *down,
                                  const uint16_t *input, const int32_t *token_ids,
                                  uint16_t *output, int tokens, int experts, void *stream);

/* The ordered combine on its own: out[t] = bf16(acc + bf16(y[p] * w)) over
 * token t's routes p = route_pos[t][k] (rows of y in route order, -1 = a
 * dropped route) in ascending p, w = scores[t][k] (BF16), then
 * + bf16(sig[t] * shared_rows[t]) when shared_rows != NULL; top_k <= 16.
 * Replaces _ordered_sum (edge35b/fused_experts.py:27-37) and _combine
 * (edge35b/block_experts.py:31-49), the index_add_ of
 * modeling_qwen3_5_moe.py:749-750 and the gated add of :788-790.
 *
 * The shared expert on its own (modeling_qwen3_5_moe.py:698-711, :779):
 * out[t] = down(bf16(silu(bf16(gate . x_t))) * bf16(up . x_t)) in BF16 with
 * FP32 accumulation, and with gate_w != NULL sig[t] = bf16(sigmoid(x_t .
 * gate_w)); gate/up [inner, hidden], down [hidden, inner]; tokens <= 128;
 * workspace of moe_shared_expert_workspace_bytes(tokens, inner). */
int moe_combine(const uint16_t *y, const int32_t *route_pos, const uint16_t *scores, const uint16_t *shared_rows,
                const uint16_t *sig, int tokens, int top_k, int hidden, uint16_t *out, void *stream);
size_t moe_shared_expert_workspace_bytes(int tokens, int inner);
int moe_shared_expert(const uint16_t *x, const uint16_t *gate, const uint16_t *up, const uint16_t *down,
                      const uint16_t *gate_w, int tokens, int hidden, int inner, uint16_t *out, uint16_t *sig,
                      void *workspace, size_t workspace_bytes, void *stream);

/* 1 when the grouped expert kernel runs as CTA pairs (tcgen05 cta_group::2,
 * 256 weight rows per product) at this width -- tokens of a layer, rows of
 * an expert-parallel owner -- on the current device, else 0.  Pairs run only
 * with LRB_GROUPED_PAIRS=1 in the environment; the results are the same bit
 * for bit either way.  No counterpart in the reference. */
int moe_grouped_paired(int tokens, int inner, int hidden);

/* ------------------------------------------------------------------------
 * One MoE layer.  moe_layer_forward replaces Qwen3_5MoeSparseMoeBlock.forward
 * (modeling_qwen3_5_moe.py:781-792: router + shared expert + experts + gate)
 * and, with route_in != NULL, Qwen3_5MoeExperts.forward as patched by
 * edge35b/expert_stream.py:457-526 (_Layer.forward :383-454; fused_forward,
 * edge35b/fused_experts.py:40-70; grouped_block, edge35b/block_experts.py:89-139):
 * the caller then supplies idx [T,top_k] and BF16 weights [T,top_k] and the
 * router and shared expert are skipped.
 * ------------------------------------------------------------------------ */
typedef struct moe_layer_weights {
    const uint16_t *router;        /* [E,H]                                   */
    const float *router_bias;      /* [E] FP32 or NULL                        */
    const uint16_t *gate_up;       /* expert e at gate_up + e*gate_up_stride: [2I,H] */
    const uint16_t *down;          /* expert e at down + e*down_stride: [H,I]  */
    int64_t gate_up_stride;        /* elements between experts (2I*H packed)  */
    int64_t down_stride;           /* elements between experts (H*I packed)   */
    const uint16_t *shared_gate;   /* [Is,H] or NULL: no shared expert        */
    const uint16_t *shared_up;     /* [Is,H]                                  */
    const uint16_t *shared_down;   /* [H,Is]                                  */
    const uint16_t *shared_gate_w; /* [H]                                     */
    int experts, hidden, inner, shared_inner, top_k;
} moe_layer_weights;

/* Optional inputs/outputs of moe_layer_forward (any pointer may be NULL). */
typedef struct moe_layer_io {
    const int64_t *route_in;       /* [T,top_k] given expert ids: skip router and shared expert */
    const uint16_t *weights_in;    /* [T,top_k] BF16 router weights for route_in */
    int64_t *idx_out;              /* [T,top_k] selected ids                   */
    uint16_t *scores_out;          /* [T,top_k] BF16 router weights            */
    uint16_t *logits_out;          /* [T,E] BF16 router logits                 */
    /* Host-resident experts.  When host_gate_up != NULL the layer copies each
     * active expert e (ascending id) from host_gate_up + e*gate_up_stride and
     * host_down + e*down_stride -- device addresses of mapped pinned banks
     * (moe_host_register) -- into slot g (the g-th active expert) of the HBM
     * slot banks, and the expert kernels read the slots; w->gate_up/down are
     * then unused.  Only the union of selected experts crosses the host link
     * (edge35b/expert_stream.py:200-236 _PackedBuffers.gather moves the same
     * rows through a pinned staging copy).  max_slots >= min(E, T*top_k). */
    const uint16_t *host_gate_up;
    const uint16_t *host_down;
    uint16_t *gate_up_slots;       /* [max_slots,2I,H]                         */
    uint16_t *down_slots;          /* [max_slots,H,I]                          */
    int max_slots;
    /* Packed host banks.  When host_descriptors != NULL (device int64
     * [2][E][3], bank 0 gate_up, bank 1 down) the host experts are in the
     * lossless row codec of edge35b/bf16_expert_codec.py -- (packed row, base,
     * escapes), base < 0 a raw row -- and are decoded in registers on their way
     * into the slots; host_gate_up/host_down are then unused. */
    const int64_t *host_descriptors;
    /* Optional cudaEvent_t handles recorded on `stream` at the stage
     * boundaries: 0 start, 1 router done, 2 permute done, 3 host gather done,
     * 4 expert plan + token gather done, 5 experts (gate/up and down) done,
     * 6 combine done (= 5 at T <= 64, where the expert kernel combines), 7 = 6.
     * NULL
     * entries (or num_stage_events <= i) are skipped.  For live per-kernel
     * timing (the role of the NVTX ranges of edge35b/native_bench.py:30-69). */
    void *const *stage_events;
    int num_stage_events;
    /* Optional device int32: 0, or nonzero when a bounded wait inside the
     * expert kernel gave up (the results of that call are then invalid). */
    int32_t *status;
    /* Expert rows instead of the combined output (expert parallelism): with
     * route_in and top_k == 1, out[t] = token t's unweighted expert row
     * bf16(act . Wd); weights_in may be NULL and no combine runs.  Rows of
     * dropped routes (ids outside [0, E)) are left untouched. */
    int rows_mode;
    /* Expert cache over the host banks (the B200 form of edge35b/
     * expert_stream.py:132-174 ExpertPool._expert's device-row LRU): with
     * expert_cache != NULL the max_slots slot banks keep experts across calls
     * and only the missing experts cross the host link.  expert_cache is
     * device int32 [E + 2*max_slots + 3], zero-filled except slot_of[0..E) and
     * expert_of[E..E+max_slots) = -1 before the first call, then owned by the
     * layer (one cache per layer and stream); the last three words count the
     * calls, the routed-expert uses and the misses.  Misses take the least
     * recently used slots; max_slots <= 1024. */
    int32_t *expert_cache;
} moe_layer_io;

/* Scratch bytes moe_layer_forward needs for `tokens` tokens. */
size_t moe_layer_workspace_bytes(int tokens, int experts, int top_k, int hidden, int inner,
                                 int shared_inner);

/* hidden in {1024,2048,4096}, inner in {256,512,1024}, experts <= 1024,
 * top_k <= 16, shared_inner == inner.  x, out [T,H] BF16. */
int moe_layer_forward(const moe_layer_weights *w, const uint16_t *x, int tokens, uint16_t *out,
                      const moe_layer_io *io, void *workspace, size_t workspace_bytes,
                      void *stream);

/* ------------------------------------------------------------------------
 * Descriptor-driven expert gathers.  Same tables and semantics as the kernels
 * of edge35b/bf16_gather_ada.cu (ABI :105-107, bound through NVRTC +
 * cuLaunchKernel by edge35b/native_bf16_gather.py:71-77 NativeBf16Gather.copy):
 *   descriptors int64 [banks][experts][3], destinations int64 [banks]
 *   (device addresses), sizes int64 [banks] (row bytes), source_ids /
 *   destination_ids int32 [max_copies], count int64 [1] read on the device.
 * Row r < *count copies expert source_ids[r] of every bank into slot
 * destination_ids[r] of that bank's destination.
 *   codec MOE_CODEC_ROW      (src, base, escapes): base < 0 copies raw bytes,
 *                            else the row codec of edge35b/bf16_expert_codec.py
 *                            (gather_bf16 / gather_bf16_l2, :36-115);
 *   codec MOE_CODEC_TILES    (packed, bases, raw): bases == 0 copies raw, else
 *                            256-value tiles of cpu_bf16_reads.h:16-52
 *                            (gather_bf16_cpu_tiles, :117-189);
 *   codec MOE_CODEC_RESIDENT as TILES, and raw == -1 marks a compact row with
 *                            uint32 headers (gather_bf16_resident, :191-198;
 *                            edge35b/gpu_resident_experts.py:22-42 encode).
 * Sources may be device memory or mapped pinned host memory.  stripes splits a
 * row across CTAs (geometry of native_bf16_gather.py:7-11); threads per CTA is
 * a multiple of 32 in [32,1024].  Rows need row_bytes % 16 == 0 (raw/row codec)
 * or % 512 == 0 (tile codecs); every 16-byte unit is written whatever the
 * stripe count.
 * ------------------------------------------------------------------------ */
#define MOE_CODEC_ROW 0
#define MOE_CODEC_TILES 1
#define MOE_CODEC_RESIDENT 2
#define MOE_CODEC_ROW_L2 3 /* MOE_CODEC_ROW with L2-only loads (gather_bf16_l2) */

int moe_gather_rows(const int64_t *descriptors, const int64_t *destinations,
                    const int64_t *sizes, const int32_t *source_ids,
                    const int32_t *destination_ids, const int64_t *count, int experts,
                    int banks, int max_copies, int codec, int stripes, int threads,
                    void *stream);

/* ------------------------------------------------------------------------
 * Packed primary cache.  Replaces edge35b/bf16_gather_ada.cu stage_bf16_primary
 * (:202-308, bound by native_bf16_gather.py:79-84 stage_primary) and
 * gather_bf16_compact_tail (:312-381, native_bf16_gather.py:86-93).  Slots hold
 * rows in the compact tile codec (tile t at t*384 + 128 * raw tiles before t);
 * prefix_tables[bank] -> uint64 [E][tiles/32] = (raw tiles before the group
 * << 32) | raw-tile bitmask.  Rows are multiples of 16384 bytes.
 *
 * moe_stage_primary: for row r < *count of plan (int32 [3][max_rows]: expert,
 *   slot, miss) and every bank b, with layouts[b] = (packed slot base, raw slot
 *   base, work rows base, packed slot stride, row bytes): a packed slot
 *   (0 <= slot < packed_slots) is decoded into work row r+1 on a hit and, on a
 *   miss, read from sources[b][expert] (tile codec: packed, bases, raw) or
 *   miss_sources[b][expert] (a compact replica, raw == -1, or a raw replica,
 *   bases == 0) into work row r+1 while its compact bytes refill the slot; a
 *   raw slot (slot >= packed_slots) is filled on a miss and skipped on a hit;
 *   slot < 0 stages into the work row only.
 * moe_gather_compact_tail: row r writes the BF16 row of expert source_ids[r]
 *   to destinations[b] + dest_ids[r] * sizes[b]; entries (int32 [2][max_rows]:
 *   tail entry or -1, resident flag) select a tail entry at tail[b] = (base,
 *   stride): a resident row is decoded from its entry, a miss with an entry
 *   also writes the entry's compact bytes.
 * ------------------------------------------------------------------------ */
int moe_stage_primary(const int64_t *sources, const int64_t *miss_sources, const int64_t *layouts,
                      const int64_t *prefix_tables, const int32_t *plan, const int32_t *count,
                      int experts, int packed_slots, int max_rows, int banks, void *stream);
int moe_gather_compact_tail(const int64_t *sources, const int64_t *destinations,
                            const int64_t *sizes, const int64_t *prefix_tables,
                            const int64_t *tail, const int32_t *source_ids,
                            const int32_t *dest_ids, const int64_t *count,
                            const int32_t *entries, const int64_t *resident, int experts,
                            int max_rows, int banks, void *stream);

/* ------------------------------------------------------------------------
 * Lossless codec encoders on the device.  The same bytes as the host encoders
 * the gather kernels decode:
 *
 * moe_rowcodec_plan replaces edge35b/bf16_expert_codec.py:26-33
 *   exponent_window + :66-78 plan_bank for a bank of `rows` rows of n BF16
 *   values (n a multiple of 8, bank 16-byte aligned): meta (int64 [rows][3])
 *   = (packed offset, or -1 for a row kept raw because its escapes exceed 1%
 *   of n; window base; escapes), *total = packed bytes (offsets and sizes
 *   rounded up to 16 bytes).
 * moe_rowcodec_pack replaces :40-51 pack_row over every packed row of that
 *   plan: [n sign|fraction bytes][n/2 exponent-delta nibbles][int32 escape
 *   indices, ascending][uint16 escape values] at packed + offset.
 * Both take a device workspace of moe_rowcodec_workspace_bytes(rows, n)
 *   bytes, the same one: pack reads the per-chunk exponent histograms that
 *   plan left there, so the bank is read twice in all (histograms, pack).
 * moe_tilecodec_pack replaces edge35b/cpu_bf16_reads.h:16-52
 *   pack_cpu_read_tiles: per 256-value tile, bases[t] = the smallest 7-bit
 *   exponent when the tile's exponents span at most 8 (else 255, raw, its 384
 *   packed bytes zeroed); packed + 384 t = 256 low bytes + 128 bytes of 4-bit
 *   codes.  *encoded (device uint64, not cleared) += tiles encoded.
 * moe_tilecodec_compact replaces the compact-row assembly of
 *   edge35b/gpu_resident_experts.py:22-42 encode (after pack_cpu_read_tiles):
 *   for `rows` rows of tiles_per_row tiles each (raw [rows][tiles*256],
 *   packed / bases from moe_tilecodec_pack of the same rows), a row r with
 *   data_offsets[r] >= 0 gets at arena + data_offsets[r] its tiles back to
 *   back -- 384 packed bytes per encoded tile, the 512 source bytes of a raw
 *   one -- and at arena + header_offsets[r] one uint32 per tile, (raw tiles
 *   before it << 8) | base; sizes[r] = its data bytes.  A row whose data or
 *   headers would leave [0, arena_bytes) or start off a 16-byte boundary gets
 *   sizes[r] = -1 and is not written; data_offsets[r] < 0 skips the row
 *   (sizes[r] = 0).  data_offsets, header_offsets, sizes: device int64 [rows].
 * ------------------------------------------------------------------------ */
size_t moe_rowcodec_workspace_bytes(int rows, int64_t n);
int moe_rowcodec_plan(const uint16_t *bank, int rows, int64_t n, int64_t *meta, int64_t *total, void *workspace,
                      size_t workspace_bytes, void *stream);
int moe_rowcodec_pack(const uint16_t *bank, int rows, int64_t n, const int64_t *meta, uint8_t *packed,
                      void *workspace, size_t workspace_bytes, void *stream);
int moe_tilecodec_pack(const uint16_t *raw, int64_t tiles, uint8_t *packed, uint8_t *bases,
                       unsigned long long *encoded, void *stream);
int moe_tilecodec_compact(const uint16_t *raw, const uint8_t *packed, const uint8_t *bases, int rows,
                          int64_t tiles_per_row, uint8_t *arena, int64_t arena_bytes, const int64_t *data_offsets,
                          const int64_t *header_offsets, int64_t *sizes, void *stream);

/* ------------------------------------------------------------------------
 * Expert parallelism (no counterpart in the reference, which runs its MoE
 * layer on one GPU).  Rank r of `world` owns experts [r*E/world, (r+1)*E/world);
 * the exchange between these calls is NCCL all_to_all_single.
 *
 * moe_ep_dispatch: after moe_router_topk + moe_permute of the rank's own tokens,
 *   send_rows[p] = x[perm_token[p]] (BF16 [T*top_k, hidden]) and
 *   send_meta[p] = the local expert id on the owning rank, for every valid
 *   route position p (in the permuted order, which is grouped by destination
 *   rank); send_counts[d] (int64 [world]) = routes owned by rank d.
 * moe_ep_unpack: received ids -> route_in (int64 [rows, 1]) of a one-slot
 *   moe_layer_forward in rows_mode over the rank's local experts, whose output
 *   row i is the unweighted expert row y_i.
 * moe_ep_combine: the layer's ordered combine over rows returned in the
 *   permuted order: out[t] = bf16(acc + bf16(ret[p] * w)) over t's routes p =
 *   route_pos[t][k] in ascending p, w = scores[t][k] (BF16), then
 *   + bf16(sig[t] * shared_rows[t]) (shared_rows may be NULL).  top_k <= 16.
 * ------------------------------------------------------------------------ */
int moe_ep_dispatch(const uint16_t *x, const int64_t *idx,
                    const int32_t *offsets, const int32_t *perm_token, const int32_t *perm_slot,
                    int tokens, int top_k, int experts, int hidden, int world,
                    uint16_t *send_rows, int32_t *send_meta, int64_t *send_counts, void *stream);
int moe_ep_unpack(const int32_t *meta, int rows, int64_t *route_in, void *stream);
int moe_ep_combine(const uint16_t *ret, const int32_t *route_pos, const uint16_t *scores,
                   const uint16_t *shared_rows, const uint16_t *sig, int tokens, int top_k,
                   int hidden, uint16_t *out, void *stream);

/* ------------------------------------------------------------------------
 * Expert-parallel step over NVLink peer memory, with the exchange fused into
 * the expert kernel (no host synchronisation; no counterpart in the
 * reference).  Every rank allocates one symmetric buffer with moe_ipc_alloc
 * (zero-filled; the 64-byte handle goes to the peers, which map it with
 * moe_ipc_open) holding, at the byte offsets below: flags_publish
 * uint32[world], flags_return uint32[world], count int32[world], meta
 * int32[world][capacity][4], tokens BF16[own_rows][hidden] (the rank's own
 * token rows) and ret BF16[capacity][hidden]; capacity >= own_rows * top_k,
 * own_rows >= the tokens of any step, offsets of tokens, meta and ret
 * 16-byte aligned.  `peers` lists every rank's buffer as mapped in this
 * process (its own included); step (uint32, start at 1), sync (int32[66],
 * zero) and error are this rank's device words.  One step:
 *   moe_ep_p2p_route    the layer's router over the rank's own tokens (the
 *                       outputs of moe_router_topk_ws: logits, idx, BF16
 *                       scores, sig; workspace of
 *                       moe_ep_p2p_route_workspace_bytes, or NULL for the
 *                       unsplit logits), copies x into tokens, gives route
 *                       (t, k) the return row route_pos[t][k] = t * top_k +
 *                       (rank of its expert among the token's top_k) and
 *                       writes one entry (local expert, return row, token)
 *                       per route into the owning rank's meta (owner and
 *                       local index from `placement`), then releases
 *                       its flags_publish; no token row crosses a link here
 *                       and no permute is needed;
 *   moe_ep_p2p_experts  on the owner: waits for every sender, plans one group
 *                       per local expert with routes plus the shared expert
 *                       over the own tokens, then runs the grouped tensor-core
 *                       kernel, which pulls each row from its sender's tokens
 *                       over NVLink and stores its down row into the sender's
 *                       ret (the shared expert's rows into shared_rows
 *                       [tokens, hidden]); gate_up [El+1, 2I, H] and down
 *                       [El+1, H, I] hold the local experts, then the shared
 *                       expert; stats (or NULL): int32 [2 + world] = rows
 *                       received, local experts with rows, rows per sender;
 *                       kernel_events (or NULL): two cudaEvent_t recorded
 *                       around the grouped kernel;
 *   moe_ep_p2p_finish   releases every sender's flags_return, waits for every
 *                       owner's, advances *step;
 *   moe_ep_combine      over ret, route_pos, scores, shared_rows and sig (a
 *                       token's routes summed in ascending return row, i.e.
 *                       ascending expert id).
 * Waits give up (1 s for the flags, 2 s inside the expert kernel) with
 * *error = 1 (publish), 2 (return) or 3 (expert kernel), and 4 when the
 * placement table names an owner or local index out of range; the GPU is never
 * left waiting. */
typedef struct moe_ep_p2p {
    const int64_t *peers;
    int64_t off_flags_publish, off_flags_return, off_count, off_meta, off_tokens, off_ret;
    int world, rank, capacity, hidden, top_k, experts, local_experts, own_rows;
    uint32_t *step;
    int32_t *sync, *error;
    /* Expert placement (device int32[experts], or NULL): entry e = (owner rank
     * << 16) | (e's index among its owner's local experts).  NULL: rank r owns
     * experts [r * local_experts, (r + 1) * local_experts).  Every rank owns
     * local_experts experts, and every rank passes the same table. */
    const int32_t *placement;
} moe_ep_p2p;

int moe_ipc_alloc(size_t bytes, void **ptr, void *handle64);
int moe_ipc_free(void *ptr);
int moe_ipc_open(const void *handle64, void **ptr);
int moe_ipc_close(void *ptr);
size_t moe_ep_p2p_route_workspace_bytes(const moe_ep_p2p *p, int tokens);
int moe_ep_p2p_route(const moe_ep_p2p *p, const uint16_t *x, int tokens, const uint16_t *router,
                     const float *bias, const uint16_t *shared_gate_w, uint16_t *logits, int64_t *idx,
                     uint16_t *scores, uint16_t *sig, int32_t *route_pos, void *workspace,
                     size_t workspace_bytes, void *stream);
size_t moe_ep_p2p_workspace_bytes(const moe_ep_p2p *p, int inner);
int moe_ep_p2p_experts(const moe_ep_p2p *p, const uint16_t *gate_up, const uint16_t *down, int inner,
                       int tokens, uint16_t *shared_rows, int32_t *stats, void *workspace,
                       size_t workspace_bytes, void *const *kernel_events, void *stream);
int moe_ep_p2p_finish(const moe_ep_p2p *p, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* LIGHTREASON_B200_MOE_H */
