/*
 * duplex_b200.h -- C ABI of the B200 (sm_100a) int4 dequant-GEMV / fused-MoE path.
 *
 * This is the drop-in boundary for the reference's hot path
 * (thecodacus/qwen3-omni-duplex).  Every entry point takes plain device pointers,
 * sizes and a cudaStream_t (passed as void*), returns an int status
 * (DUPLEX_OK == 0), never allocates, never synchronises, and launches only on the
 * given stream, so every call can be captured in a CUDA graph.
 *
 * Weight format (unchanged from the reference's stacked buffers,
 * src/duplex/streaming/fused_packed_moe.py:68-80, 117-123):
 *   packed [E][Rs][K/8] int32   -- column i + 8m is nibble i (bits 4i..4i+3) of word m
 *   scale  [E][Rs][G]   fp16|bf16, G = ceil(K / group)
 *   zeros  [E][Rs][ceil(G/8)] int32 or NULL -- 4-bit zero point per (row, group), same
 *          nibble order along the group axis; NULL means zero point 8 everywhere,
 *          which is the reference's symmetric format (value = nibble - 8).
 * The GEMV entry points read it after a one-time repack into tile records
 * (duplex_repack_tiles).  K % 32 == 0; group 32 or 64 * 2^k; base pointers 16-byte aligned.
 *
 * Activations are fp16 or bf16 (DUPLEX_DTYPE_*), accumulation is fp32.
 */
#ifndef DUPLEX_B200_H
#define DUPLEX_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes */
#define DUPLEX_OK 0
#define DUPLEX_ERR_ARG 1          /* bad size / null pointer / unsupported combination */
#define DUPLEX_ERR_ALIGN 2        /* pointer or stride not 16-byte aligned */
#define DUPLEX_ERR_DTYPE 3        /* unsupported dtype code */
#define DUPLEX_ERR_WORKSPACE 4    /* workspace too small */
#define DUPLEX_ERR_CUDA 5         /* a CUDA runtime call failed (see duplex_last_cuda_error) */
#define DUPLEX_ERR_UNSUPPORTED 6  /* shape outside what the kernels implement */
#define DUPLEX_ERR_SCRATCH_LIMIT 7 /* problem needs more than the static scratch of a _noalloc call */

/* ---- device-side error word bits (written with atomicOr into `err`, never trap) */
#define DUPLEX_DEVERR_EXPERT 1    /* an expert id outside [0, E) was clamped to 0 */
#define DUPLEX_DEVERR_TIMEOUT 2   /* a bounded pipeline wait gave up */
#define DUPLEX_DEVERR_NONFINITE 4 /* duplex_stack_forward: a partial layer output was NaN or
                                     beyond +-2^26 and was clamped (its fixed-point sum) */
/* duplex_stack_forward also records, from this bit up, which of its waits gave up
 * first: 1 ring slot free, 2 routing plan, 3 ring slot filled, 4 grid barrier,
 * 5 drain, 6 cluster exchange. */
#define DUPLEX_DEVERR_SITE_SHIFT 8

/* ---- dtype codes */
#define DUPLEX_DTYPE_F16 0
#define DUPLEX_DTYPE_BF16 1
#define DUPLEX_DTYPE_F32 2

int duplex_version(void);
const char* duplex_error_string(int status);
int duplex_last_cuda_error(void);

/*
 * unpack4 -- reference `unpack4` (src/duplex/streaming/fused_packed_moe.py:54-65).
 * packed [rows][C] int32 -> out [rows][out_cols] int32 in [-8, 7]; out_cols <= 8*C.
 */
int duplex_unpack4(const int32_t* packed, int64_t rows, int32_t C, int32_t out_cols,
                   int32_t* out, void* stream);

/*
 * dequant -- reference `FusedPackedMoE._dequant` (fused_packed_moe.py:183-189) and
 * `dequantize_weight` (src/duplex/quant/dequant.py:40-77), zero-point generalised:
 * out[r][c] = round_out((nibble - zero) * scale[r][c / group]) with ONE rounding of
 * the exact product into out_dtype (F16 / BF16 / F32).  rows = E * R (any layout of
 * the leading dims), K columns.  scale_dtype F16 / BF16 / F32.
 */
int duplex_dequant(const int32_t* packed, const void* scale, int scale_dtype,
                   const int32_t* zeros, int64_t rows, int32_t K, int32_t group,
                   void* out, int out_dtype, void* stream);

/*
 * tile_record_bytes / repack_tiles -- the one-time weight preparation (the reference
 * restacks its experts once at module construction, fused_packed_moe.py:68-80,117-123).
 * A stacked int4 matrix in the reference layout (packed [E][R][K/8] int32, scale
 * [E][R][G] fp16|bf16, zeros [E][R][ceil(G/8)] int32 or NULL) is rewritten into one
 * record per (expert, 16-row block): fragment-ordered nibbles, pair-interleaved scales
 * and zero points, padded to 128 bytes (layout: csrc/tiles.cuh).  tiles must hold
 * E * ceil(R/16) * record_bytes bytes.  pair_halves != 0 (gate|up stacks, R % 32 == 0)
 * places row block j of the first half next to row block j of the second half.
 * K % 32 == 0; group 32 or 64 * 2^k.
 */
int duplex_tile_record_bytes(int32_t K, int32_t group, int has_zeros, size_t* bytes);
int duplex_repack_tiles(const int32_t* packed, const void* scale, const int32_t* zeros,
                        int scale_dtype, int32_t E, int32_t R, int32_t K, int32_t group,
                        int32_t pair_halves, void* tiles, size_t tiles_bytes, void* stream);

/*
 * dq_gemv -- reference `dequant_gemv` (src/duplex/streaming/triton_dequant_gemv.py:85-113).
 * out[j][r] = sum_c W[sel[j]][r][c] * x_j[c] in fp32 for r < R, W given as tiles
 * (repack_tiles with pair_halves = 0).
 * x: [K] shared by all slots (x_slot_stride = 0) or [nsel][x_slot_stride] rows.
 * sel: [nsel] int32 expert ids (device).  out: [nsel][R] fp32.
 * err: optional device int (bit DUPLEX_DEVERR_EXPERT when a sel id is out of range).
 */
int duplex_dq_gemv(const void* x, int act_dtype, int64_t x_slot_stride, const void* tiles,
                   int scale_dtype, int has_zeros, int32_t E, int32_t R, int32_t K,
                   int32_t group, const int32_t* sel, int32_t nsel, float* out, int32_t* err,
                   void* stream);

/*
 * packed_linear -- reference `TritonPackedLinear.forward` (triton_dequant_gemv.py:151-159)
 * for B <= 8 rows in one launch (the reference launches once per row):
 * y[b][r] = round_act(round_act(sum_c W[r][c] x[b][c]) + bias[r]) (+ residual[b][r], one
 * more rounding; not in the reference, used by the clock-path stack).  W as tiles (E = 1).
 * x [B][K] rows x_row_stride apart; out [B][R] rows out_row_stride apart (act dtype).
 * rms_eps > 0 first RMS-normalises each x row (x * rsqrt(mean(x^2) + rms_eps), rounded to the
 * act dtype; a weightless RMSNorm, used by the clock-path stack), rms_eps <= 0 leaves x as is.
 * pdl != 0 launches with programmatic dependent launch and prefetches the weights
 * before waiting on the previous kernel.
 */
int duplex_packed_linear(const void* x, int act_dtype, int32_t B, int64_t x_row_stride,
                         const void* tiles, int scale_dtype, int has_zeros, int32_t R,
                         int32_t K, int32_t group, const void* bias, const void* residual,
                         int64_t res_row_stride, void* out, int64_t out_row_stride,
                         float rms_eps, int pdl, void* stream);

/*
 * moe_workspace_bytes -- bytes of scratch the MoE entry points need for T tokens.
 */
int duplex_moe_workspace_bytes(int32_t T, int32_t E, int32_t H, int32_t I, int32_t top_k,
                               size_t* bytes);

/*
 * moe_route -- router of `FusedPackedMoE.forward` (fused_packed_moe.py:195-199):
 * logits = x @ gate_w^T (+ gate_b), rounded to the act dtype (nn.Linear in the module
 * dtype), softmax in fp32, top-k (ties -> lower expert id), renormalised when
 * norm_topk != 0.  x [T][H], gate_w [E][H] (act dtype), gate_b [E] or NULL.
 * w_out [T][top_k] fp32, sel_out [T][top_k] int32.  T <= 8, E <= 256, top_k <= 8.
 * workspace: duplex_moe_workspace_bytes bytes, zero-filled once before first use.
 * rms_eps > 0 routes the RMS-normalised tokens (as packed_linear) and leaves them in the
 * workspace for the expert kernels.
 */
int duplex_moe_route(const void* x, int act_dtype, int32_t T, const void* gate_w,
                     const void* gate_b, int32_t E, int32_t H, int32_t top_k,
                     int32_t norm_topk, float* w_out, int32_t* sel_out, void* workspace,
                     size_t workspace_bytes, float rms_eps, int pdl, void* stream);

/*
 * moe_forward -- the whole of `FusedPackedMoE.forward` (fused_packed_moe.py:191-275) for
 * T <= 8 tokens: route -> gate|up dequant-GEMV with SiLU(gate)*up epilogue -> down
 * dequant-GEMV with the routing-weighted combine epilogue, three launches chained by
 * programmatic dependent launch when pdl != 0.  Tokens that pick the same expert
 * share one pass over its weights.
 * gu_tiles: repack_tiles of [E][2I][H/8] (gate rows 0..I-1, up rows I..2I-1) with
 * pair_halves = 1; dn_tiles: repack_tiles of [E][H][I/8].  Same group and zero-point use.
 * out [T][H] act dtype (+ residual [T][H] when not NULL, fp32 add).  w_out/sel_out as in
 * moe_route (may be NULL).  err: optional device int.  rms_eps > 0: the experts see the
 * RMS-normalised tokens, the residual is added to the un-normalised output.
 */
int duplex_moe_forward(const void* x, int act_dtype, int32_t T, const void* gate_w,
                       const void* gate_b, int32_t E, int32_t H, int32_t I, int32_t top_k,
                       int32_t norm_topk, const void* gu_tiles, const void* dn_tiles,
                       int scale_dtype, int has_zeros, int32_t group, const void* residual,
                       void* out, float* w_out,
                       int32_t* sel_out, void* workspace, size_t workspace_bytes,
                       int32_t* err, float rms_eps, int pdl, void* stream);

/*
 * Host-resident experts -- the reference's `FusedPackedMoE(host_resident=True)` layers
 * (fused_packed_moe.py:130-164 staging blobs, :233-253 per-token copies).
 * host_alloc: mapped pinned host memory (cudaHostAllocMapped | cudaHostAllocPortable);
 * *host_ptr is for host code, *dev_ptr the address kernels read it at.  host_free
 * releases it (host pointer).
 * moe_forward_staged: duplex_moe_forward with the expert tile records (same layout)
 * in host memory: gu_tiles_host / dn_tiles_host are DEVICE addresses of mapped pinned
 * memory (host_alloc's dev_ptr).  The router writes the unit plan, one kernel copies
 * the records of the planned experts from host memory into the slots of `stage`
 * (duplex_moe_stage_bytes), and the expert kernels run on the slots: no host
 * synchronisation, bit-identical output to duplex_moe_forward on resident records.
 * The expert kernels follow the router in plain stream order (pdl applies to the
 * router only).  One call at a time per stage buffer and per workspace.
 */
int duplex_host_alloc(size_t bytes, void** host_ptr, void** dev_ptr);
int duplex_host_free(void* host_ptr);
int duplex_moe_stage_bytes(int32_t T, int32_t E, int32_t H, int32_t I, int32_t top_k,
                           int32_t group, int has_zeros, size_t* bytes);
int duplex_moe_forward_staged(const void* x, int act_dtype, int32_t T, const void* gate_w,
                              const void* gate_b, int32_t E, int32_t H, int32_t I,
                              int32_t top_k, int32_t norm_topk, const void* gu_tiles_host,
                              const void* dn_tiles_host, int scale_dtype, int has_zeros,
                              int32_t group, const void* residual, void* out, float* w_out,
                              int32_t* sel_out, void* workspace, size_t workspace_bytes,
                              void* stage, size_t stage_bytes, int32_t* err, float rms_eps,
                              int pdl, void* stream);

/*
 * moe_grouped_workspace_bytes -- scratch of duplex_moe_grouped for T tokens (logits,
 * selection, the expert-sorted assignment list, the unit list and one fp32 output row
 * per (token, slot)).  No zero fill needed.  Returns DUPLEX_ERR_UNSUPPORTED for a
 * geometry the grouped path does not take (see duplex_moe_grouped), so it doubles as
 * the support query.
 */
int duplex_moe_grouped_workspace_bytes(int32_t T, int32_t E, int32_t H, int32_t I,
                                       int32_t top_k, int32_t group, int has_zeros,
                                       size_t* bytes);

/*
 * moe_grouped -- `FusedPackedMoE.forward` (fused_packed_moe.py:191-275) for a batch of
 * T <= 512 tokens (batched decode of many streams, prefill chunks), where the T <= 8
 * entry points above do not apply.  Five launches on `stream`: router logits on the
 * tensor cores (skipped when logits_in != NULL: [T][E] fp32, already rounded to the act
 * dtype), top-k + softmax, a stable counting sort of the T*top_k (token, slot) pairs by
 * expert into units of <= 20 tokens, one CTA per unit streaming its expert's gate|up and
 * down tiles once (SiLU(gate)*up kept in shared memory), and the routing-weighted
 * combine in selection order (+ residual), one rounding.  Arguments as duplex_moe_forward
 * (rms_eps and pdl excepted); E <= 256, top_k <= 8, H and I multiples of 64, group a
 * power of two >= 64, one unit's tokens, intermediate and two weight stages within
 * 227 KB of shared memory (Thinker geometry, hidden 2048 / inter 768, takes 212 KB),
 * scale dtype == act dtype.  x, out, tiles, gate_w and workspace
 * 16-byte aligned.  err: device int, DUPLEX_DEVERR_EXPERT when a selected id is out of
 * range, DUPLEX_DEVERR_TIMEOUT when a copy wait gives up (bounded, about 2 s).
 * Deterministic: every reduction runs in a fixed order (bit-identical across calls and
 * graph replays).
 */
int duplex_moe_grouped(const void* x, int act_dtype, int32_t T, const void* gate_w,
                       const void* gate_b, const float* logits_in, int32_t E, int32_t H,
                       int32_t I, int32_t top_k, int32_t norm_topk, const void* gu_tiles,
                       const void* dn_tiles, int scale_dtype, int has_zeros, int32_t group,
                       const void* residual, void* out, float* w_out, int32_t* sel_out,
                       void* workspace, size_t workspace_bytes, int32_t* err, void* stream);

/*
 * moe_route_grouped -- the router of duplex_moe_grouped alone (logits on the tensor
 * cores unless logits_in is given, fp32 softmax, top-k, renormalised) for T <= 512
 * tokens: w_out / sel_out [T][top_k] (either may be NULL when pack is given).  Same
 * numerics as duplex_moe_route (T <= 8).  pack (optional): token t's expert-parallel
 * exchange row at pack + t * pack_row_bytes -- the token (2 H bytes, copied from x), its
 * top_k expert ids (int32), its top_k weights (fp32); pack_row_bytes >= 2 H + 8 top_k, a
 * multiple of 16.  workspace: at least T * E * 4 bytes (the logits), 16-byte aligned.
 */
int duplex_moe_route_grouped(const void* x, int act_dtype, int32_t T, const void* gate_w,
                             const void* gate_b, const float* logits_in, int32_t E, int32_t H,
                             int32_t top_k, int32_t norm_topk, float* w_out, int32_t* sel_out,
                             void* pack, int64_t pack_row_bytes, void* workspace,
                             size_t workspace_bytes, int32_t* err, void* stream);

/*
 * moe_experts_grouped -- the expert half of duplex_moe_grouped for a given selection,
 * restricted to one expert-parallel rank's experts: for every token t and slot j whose
 * expert e = sel[t][j] lies in [e_begin, e_begin + E_local), y = down(SiLU(gate(x_t)) *
 * up(x_t)) with that expert's tiles (gu_tiles / dn_tiles hold the E_local local experts,
 * local index e - e_begin); out[t] = sum of w[t][j] * y over those slots in selection
 * order (+ residual[t]), rounded once to out_dtype (the act dtype, or DUPLEX_DTYPE_F32 for
 * partial sums that other ranks' partials are added to).  Slots of other ranks'
 * experts are skipped; ids outside [0, E_total) set DUPLEX_DEVERR_EXPERT and are
 * skipped.  x: T rows x_row_stride elements apart (>= H, a multiple of 8: token rows
 * packed with other per-token data, as an expert-parallel exchange delivers them).
 * sel / w: token t's top_k expert ids (int32) / weights (fp32) at sel / w + t *
 * meta_stride (4-byte words; top_k when dense, the exchange row when packed).  T <= 512;
 * the unit token
 * cap is chosen from T * top_k / E_total.  Other arguments and limits as
 * duplex_moe_grouped; workspace: duplex_moe_experts_grouped_workspace_bytes.
 */
int duplex_moe_experts_grouped_workspace_bytes(int32_t T, int32_t E_local, int32_t E_total,
                                               int32_t H, int32_t I, int32_t top_k,
                                               int32_t group, int has_zeros, size_t* bytes);
int duplex_moe_experts_grouped(const void* x, int act_dtype, int32_t T, int64_t x_row_stride,
                               const int32_t* sel, const float* w, int32_t meta_stride,
                               int32_t top_k, int32_t e_begin, int32_t E_local,
                               int32_t E_total, int32_t H, int32_t I, const void* gu_tiles,
                               const void* dn_tiles, int scale_dtype, int has_zeros,
                               int32_t group, const void* residual, void* out, int out_dtype,
                               void* workspace, size_t workspace_bytes, int32_t* err,
                               void* stream);

/*
 * ep_dispatch_pack / ep_combine -- the two device steps around the expert-parallel
 * all-to-alls (no counterpart in the reference, which keeps every expert on one GPU,
 * fused_packed_moe.py:165-169; the expert stage between them is
 * duplex_moe_experts_grouped).  n_ranks ranks, E / n_ranks experts each.
 * dispatch_pack: rows [T][row_bytes] are this rank's exchange rows (duplex_moe_route_grouped
 * with pack: the token, its top_k expert ids (int32) at ids_offset, its top_k weights
 * (fp32) right after); for every rank d, the rows of the tokens that selected one of d's
 * experts go, compacted in token order, to block d of send ([n_ranks][T][row_bytes]);
 * rows of a block past its count get the first expert id of rank d + 1 (mod n_ranks) and
 * weight 0, which d's expert stage skips.  slot_of[d][t] = token t's row in block d, -1
 * when t was not sent to d.  T <= 512, row_bytes % 16 == 0.
 * ep_combine: out[t] = sum over d = 0 .. n_ranks - 1 of partials[d][slot_of[d][t]] (fp32
 * rows [n_ranks][T][H], as the second all-to-all returns them) (+ residual[t]), one
 * rounding to act_dtype.  H % 4 == 0.
 */
int duplex_ep_dispatch_pack(const void* rows, int64_t row_bytes, int32_t T, int32_t top_k,
                            int32_t E, int32_t n_ranks, int64_t ids_offset, void* send,
                            int32_t* slot_of, void* stream);
int duplex_ep_combine(const float* partials, const int32_t* slot_of, int32_t T, int32_t n_ranks,
                      int32_t H, const void* residual, void* out, int act_dtype, void* stream);

/*
 * Peer exchange of the expert-parallel layer over NVLink (the NCCL all-to-alls' stand-in):
 * buffers allocated with ipc_alloc (cudaMalloc, zero-filled, with a CUDA IPC handle of
 * ipc_handle_bytes() bytes), shared through the host's process group and opened on every
 * other rank with ipc_open (plain peer mappings: no NVLink multicast object).
 * ep_dispatch_peer is ep_dispatch_pack writing block d straight into destination d's
 * receive buffer (recv_peers[d], at block `rank`); ep_put_peer copies block d of `src`
 * (n_ranks blocks of block_bytes) into dst_peers[d] at block `rank`.  Both end with the
 * last CTA writing the exchange's epoch (counted in `epoch`, local) into slot `rank` of
 * every destination's flag array (flag_peers[d]); ep_wait waits on this rank's own
 * flag array until every slot holds the epoch, bounded by wait_limit_cycles (<= 0:
 * about 2 s), after which it sets DUPLEX_DEVERR_TIMEOUT and returns instead of hanging.
 * recv_peers / dst_peers / flag_peers are DEVICE arrays of n_ranks pointers.
 */
int duplex_ipc_handle_bytes(void);
int duplex_ipc_alloc(size_t bytes, void** ptr, void* handle);
int duplex_ipc_open(const void* handle, void** ptr);
int duplex_ipc_close(void* ptr);
int duplex_ipc_free(void* ptr);
int duplex_ep_dispatch_peer(const void* rows, int64_t row_bytes, int32_t T, int32_t top_k,
                            int32_t E, int32_t n_ranks, int32_t rank, int64_t ids_offset,
                            void* const* recv_peers, int32_t* slot_of,
                            unsigned* const* flag_peers, unsigned* counter, unsigned* epoch,
                            void* stream);
int duplex_ep_put_peer(const void* src, int64_t block_bytes, int32_t n_ranks, int32_t rank,
                       void* const* dst_peers, unsigned* const* flag_peers, unsigned* counter,
                       unsigned* epoch, void* stream);
int duplex_ep_wait(const unsigned* flags, const unsigned* epoch, int32_t n_ranks,
                   int64_t wait_limit_cycles, int32_t* err, void* stream);

/*
 * talker_moe_forward -- the Talker's MoE block, `FusedMoE.forward` of the reference
 * (src/duplex/streaming/fused_moe.py:40-141), for T <= 8 tokens: router (as moe_route),
 * the selected experts' gate|up with SiLU(gate) * up, down, the routing-weighted sum over
 * the slots in selection order, plus the shared expert gated by
 * sigmoid(x . sh_gate_w) (fused_moe.py:136-140), with the reference's rounding to the
 * act dtype after each of those steps.  gate_up [E][2I][H] (gate rows, then up rows),
 * down [E][H][I]: act dtype, or int8 (weight_int8 != 0) with per-row scales
 * gu_scale [E][2I] and dn_scale [E][H] in the act dtype, a weight being round(q * s)
 * (the reference's q8 format, fused_moe.py:84-97).  Shared expert (optional: sh_gate
 * NULL): sh_gate / sh_up [S][H], sh_down [H][S], sh_gate_w [H] or NULL (gate 1), act
 * dtype.  H, I, S multiples of 8 (of 16 for int8 rows); pointers 16-byte aligned.
 * w_out / sel_out [T][top_k] or NULL.  workspace: duplex_talker_moe_workspace_bytes,
 * zero-filled once before first use.  err: DUPLEX_DEVERR_EXPERT for an out-of-range id.
 */
int duplex_talker_moe_workspace_bytes(int32_t T, int32_t E, int32_t H, int32_t I, int32_t top_k,
                                      int32_t S, size_t* bytes);
int duplex_talker_moe_forward(const void* x, int act_dtype, int32_t T, const void* gate_w,
                              int32_t E, int32_t H, int32_t I, int32_t top_k, int32_t norm_topk,
                              const void* gate_up, const void* down, int weight_int8,
                              const void* gu_scale, const void* dn_scale, const void* sh_gate,
                              const void* sh_up, const void* sh_down, int32_t S,
                              const void* sh_gate_w, void* out, float* w_out, int32_t* sel_out,
                              void* workspace, size_t workspace_bytes, int32_t* err, void* stream);

/*
 * Tensor-core (tcgen05) variants of the grouped path -- same computation, arguments,
 * limits and error behaviour as duplex_moe_grouped / duplex_moe_experts_grouped, with
 * the experts in "tensor-core records" instead of tile records, and these limits: group
 * 128, H and I multiples of 128 and at least 256.  The weights are dequantised exactly
 * as the reference's dequant does ((nibble - zero) * scale, one rounding into the
 * activation type) straight into tensor memory and multiplied on the tensor cores with
 * fp32 accumulation; units hold up to 16, 32 or 64 tokens (chosen from T * top_k /
 * E_total).  Deterministic (fixed accumulation order), but not bit-identical to the
 * mma.sync path, whose weights are not rounded.
 *
 * tc_records_bytes -- size of the records of a stacked matrix [E][R][K/8] (R a multiple of
 * 128; pair_halves for gate|up, R = 2 I).  repack_tc_records -- build them from the
 * reference's tensors (packed, scale [E][R][K/128], optional packed zero points), as
 * duplex_repack_tiles does for tile records; records 16-byte aligned.
 */
int duplex_tc_records_bytes(int32_t E, int32_t R, int32_t K, int32_t group, int has_zeros,
                            int32_t pair_halves, size_t* bytes);
int duplex_repack_tc_records(const int32_t* packed, const void* scale, const int32_t* zeros,
                             int scale_dtype, int32_t E, int32_t R, int32_t K, int32_t group,
                             int32_t pair_halves, void* records, size_t records_bytes,
                             void* stream);
int duplex_moe_grouped_tc_workspace_bytes(int32_t T, int32_t E, int32_t H, int32_t I,
                                          int32_t top_k, int32_t group, int has_zeros,
                                          size_t* bytes);
int duplex_moe_grouped_tc(const void* x, int act_dtype, int32_t T, const void* gate_w,
                          const void* gate_b, const float* logits_in, int32_t E, int32_t H,
                          int32_t I, int32_t top_k, int32_t norm_topk, const void* gu_records,
                          const void* dn_records, int scale_dtype, int has_zeros, int32_t group,
                          const void* residual, void* out, float* w_out, int32_t* sel_out,
                          void* workspace, size_t workspace_bytes, int32_t* err, void* stream);
int duplex_moe_experts_grouped_tc_workspace_bytes(int32_t T, int32_t E_local, int32_t E_total,
                                                  int32_t H, int32_t I, int32_t top_k,
                                                  int32_t group, int has_zeros, size_t* bytes);
int duplex_moe_experts_grouped_tc(const void* x, int act_dtype, int32_t T, int64_t x_row_stride,
                                  const int32_t* sel, const float* w, int32_t meta_stride,
                                  int32_t top_k, int32_t e_begin, int32_t E_local,
                                  int32_t E_total, int32_t H, int32_t I, const void* gu_records,
                                  const void* dn_records, int scale_dtype, int has_zeros,
                                  int32_t group, const void* residual, void* out, int out_dtype,
                                  void* workspace, size_t workspace_bytes, int32_t* err,
                                  void* stream);

/*
 * Persistent clock-path stack -- the reference's clock path (src/duplex/streaming/clock.py:
 * 162-197) runs Thinker layers 0..23 per frame with TritonPackedLinear q/k/v/o and
 * FusedPackedMoE; this is every int4 linear of n_layers such layers for T <= 8 tokens in ONE
 * launch: per layer q|k|v of rms(h), o of q (+ h) -> h1, router / top-k / plan on rms(h1),
 * gate|up + SiLU, down + combine (+ h1 when moe_residual) -> next h.  With has_attn == 0 a
 * layer is only the MoE (x -> MoE(rms(x)) (+ x)).  `layers` is a DEVICE array of n_layers
 * descriptors: q|k|v [qkv_R][H] and o [H][q_dim] tiles and the gate|up tiles (pair_halves)
 * from duplex_repack_tiles, in gate_w the router's gate matrix as gate records from
 * duplex_repack_gate_records (+ gate_b [E] in the act dtype), and in dn_tiles the down
 * projection as K-slice records from duplex_repack_down_slices.  The attention
 * core is not part of it: o reads the first q_dim outputs of q|k|v.
 * Limits: H a multiple of 128 and <= 4096, I a multiple of 128, q_dim a multiple of 64,
 * group 32, 64 or 128, scale dtype == act dtype.
 * The launch is in clusters of 8 CTAs (one CTA per SM, as many clusters as can be resident
 * at once): each MoE layer has one grid-wide barrier, the other hand-offs stay inside a
 * cluster.  It expects the GPU's SMs to itself while it runs: a CTA that cannot start
 * in time makes the grid barrier give up (DUPLEX_DEVERR_TIMEOUT), it never hangs.  workspace: duplex_stack_workspace_bytes; one call at a time per workspace
 * (the grid barrier counter in it is zeroed by a memset issued before the launch).
 * err is required: a bounded wait that gives up sets DUPLEX_DEVERR_TIMEOUT (and the
 * site of the first one from DUPLEX_DEVERR_SITE_SHIFT) instead of hanging, and while
 * that bit stays set later launches give up at once.  wait_limit_cycles: the bound of
 * every wait in SM clock cycles (<= 0: about 2 s).  test_flags: 0; bit 0 makes the first
 * grid barrier wait for one arrival more than the grid makes, so that it gives up (the
 * timeout path's test).  Bit-identical results run to run.
 */
typedef struct duplex_stack_layer {
  const void* qkv_tiles;
  const void* o_tiles;
  const void* gate_w;
  const void* gate_b;
  const void* gu_tiles;
  const void* dn_tiles;
} duplex_stack_layer;

int duplex_stack_workspace_bytes(int32_t T, int32_t H, int32_t E, int32_t I, int32_t top_k,
                                 int32_t qkv_R, size_t* bytes);
int duplex_stack_forward(const duplex_stack_layer* layers, int32_t n_layers, int32_t has_attn,
                         int32_t moe_residual, const void* x_in, void* out, int act_dtype,
                         int scale_dtype, int has_zeros, int32_t T, int32_t H, int32_t E,
                         int32_t I, int32_t top_k, int32_t norm_topk, int32_t qkv_R,
                         int32_t q_dim, int32_t group, float rms_eps, void* workspace,
                         size_t workspace_bytes, int64_t wait_limit_cycles, int32_t test_flags,
                         int32_t* err, void* stream);

/*
 * down_slices_bytes / repack_down_slices -- the down projection's layout for
 * duplex_stack_forward, built once from the reference's stacked down tensors (packed
 * [E][H][I/8] int32, scale [E][H][I/group], zeros [E][H][ceil(G/8)] or NULL; the
 * reference stacks them at fused_packed_moe.py:117-123): one record per (expert, 128-column
 * slice of I, 16 rows of H) in the tile-record layout with K = 128, padded to 16 bytes,
 * ordered [E][I/128][H/16].  group 32, 64 or 128; H a multiple of 16, I of 128.
 */
/*
 * gate_records_bytes / repack_gate_records -- the router's gate matrix (nn.Linear weight
 * [E][H], fp16 or bf16, as the reference's FusedPackedMoE.gate holds it,
 * fused_packed_moe.py:112) for duplex_stack_forward: per block of 16 experts and
 * 16-column step, the 32 lanes' mma.sync A fragments (512 bytes), rows past E zero.
 * H a multiple of 16.
 */
int duplex_gate_records_bytes(int32_t E, int32_t H, size_t* bytes);
int duplex_repack_gate_records(const void* gate_w, int dtype, int32_t E, int32_t H, void* out,
                               size_t out_bytes, void* stream);

int duplex_down_slices_bytes(int32_t E, int32_t H, int32_t I, int32_t group, int has_zeros,
                             size_t* bytes);
int duplex_repack_down_slices(const int32_t* packed, const void* scale, const int32_t* zeros,
                              int scale_dtype, int32_t E, int32_t H, int32_t I, int32_t group,
                              void* out, size_t out_bytes, void* stream);

/*
 * moe_forward_noalloc -- no counterpart in the reference.  Same computation and
 * arguments as duplex_moe_forward, minus the workspace: for callers that cannot
 * call cudaMalloc (a real-time frame loop, where an allocation can synchronise the
 * device and miss the frame deadline, or a C host without a caching allocator).
 * The scratch is a file-scope device array of duplex_moe_noalloc_scratch_bytes()
 * (1.25 MiB) per GPU, kept until the process exits; problems that need more
 * (duplex_moe_workspace_bytes larger than that) return DUPLEX_ERR_SCRATCH_LIMIT.
 * The first call on a device looks the array's address up (make it before any
 * stream capture).  All calls share the array: calls that overlap on the GPU race
 * and must be serialised by the caller.  Nothing is allocated.
 */
size_t duplex_moe_noalloc_scratch_bytes(void);
int duplex_moe_forward_noalloc(const void* x, int act_dtype, int32_t T, const void* gate_w,
                               const void* gate_b, int32_t E, int32_t H, int32_t I,
                               int32_t top_k, int32_t norm_topk, const void* gu_tiles,
                               const void* dn_tiles, int scale_dtype, int has_zeros,
                               int32_t group, const void* residual, void* out, float* w_out,
                               int32_t* sel_out, int32_t* err, float rms_eps, int pdl,
                               void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DUPLEX_B200_H */
