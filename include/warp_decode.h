/*
 * warp_decode_b200 — C ABI for the fused MoE decode kernels on B200 (sm_100a).
 *
 * This header is the drop-in boundary.  Every entry point takes plain device
 * pointers, sizes and a CUDA stream handle (passed as `void*`, i.e. the value
 * of a `cudaStream_t`; NULL means the legacy default stream).  No entry point
 * synchronises the stream or depends on PyTorch, and only wd_tp_comm_create
 * allocates device memory (the tensor-parallel exchange buffer); the kernels'
 * other global memory is the caller's (h_buf, sync) or, for
 * wd_moe_ffn_3d_batched_noalloc, a static array of the library.
 *
 * Reference interfaces replaced (Religious-J/warp_decode):
 *   wd_moe_gate_up_3d_batched  <- warp_decode::launch_moe_gate_up_3d_batched
 *                                 csrc/moe_gate_up_3d_batched.cu:117-131
 *                                 (host checks it inherits: csrc/binding.cpp:35-73)
 *   wd_moe_down_3d_batched     <- warp_decode::launch_moe_down_3d_batched
 *                                 csrc/moe_down_3d_batched.cu:124-141
 *                                 (host checks it inherits: csrc/binding.cpp:79-121)
 *   wd_moe_*_mxfp8             <- no counterpart in the reference; the MXFP8
 *                                 weight format is listed as future work in
 *                                 README.md:294-308 of the reference.
 *
 * Layouts (all row-major, contiguous):
 *   x          [B, hidden]               bf16
 *   w_gate_up  [E, 2*inter, hidden]      bf16  rows [0,inter) gate, [inter,2*inter) up
 *   topk_ids   [B, topk]                 int32
 *   h (buffer) [B*topk, inter]           bf16  h = silu(x.gate) * (x.up)
 *   w_down     [E, hidden, inter]        bf16
 *   topk_scale [B, topk]                 fp32
 *   y (out)    [B, hidden]               bf16 (or fp32 for tensor-parallel partials)
 *
 * MXFP8 weights (OCP Microscaling v1.0, MXFP8 E4M3, block size 32 along the
 * reduction axis):
 *   gate_up:  q [E, 2*inter, hidden] uint8 (e4m3), s [E, 2*inter, hidden/32] uint8 (ue8m0)
 *   down:     q [E, hidden, inter]   uint8 (e4m3), s [E, hidden, inter/32]   uint8 (ue8m0)
 *   value = e4m3(q) * 2^(s - 127)
 *
 * Error behaviour: every entry point validates its arguments on the host and
 * returns WD_OK or a wd_error_t code without launching anything on failure;
 * wd_last_error_message() then holds a human-readable reason (thread-local).
 * Device-side conditions that the host cannot see (an expert id outside
 * [0, E), a bounded wait that gave up) are OR-ed into a 32-bit status word:
 * either the caller's `status` (device pointer) or, when that is NULL, a
 * per-device word owned by the library (read it with wd_status_read).
 * Slots whose expert id is out of range contribute zeros and are never used
 * to address weight memory.
 */
#ifndef WARP_DECODE_B200_H_
#define WARP_DECODE_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__) || defined(__clang__)
#define WD_API __attribute__((visibility("default")))
#else
#define WD_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum wd_error_t {
  WD_OK = 0,
  WD_ERR_NULL_POINTER = 1,   /* a required pointer is NULL                     */
  WD_ERR_SHAPE = 2,          /* sizes are negative, zero or inconsistent        */
  WD_ERR_ALIGNMENT = 3,      /* a pointer is not 16-byte aligned                */
  WD_ERR_UNSUPPORTED = 4,    /* shape outside what the kernels implement        */
  WD_ERR_CUDA = 5            /* a CUDA runtime call or kernel launch failed     */
} wd_error_t;

/* Bits of the device status word. */
#define WD_STATUS_BAD_EXPERT_ID   0x1u  /* some topk_ids entry was outside [0, E)   */
#define WD_STATUS_WAIT_TIMEOUT    0x2u  /* a bounded pipeline wait gave up          */
#define WD_STATUS_ROUTING_CHANGED 0x4u  /* down saw topk_ids change under an early
                                           start and recomputed (informational)   */

/* Library version, as MAJOR*10000 + MINOR*100 + PATCH. */
WD_API int wd_version(void);

/* Static description of an error code. */
WD_API const char* wd_error_string(int err);

/* Detail message of the last failing call on this host thread ("" if none). */
WD_API const char* wd_last_error_message(void);

/*
 * gate_up + silu_and_mul, fused:
 *   h[b*topk+s, n] = silu(sum_k x[b,k] W[e,n,k]) * sum_k x[b,k] W[e,inter+n,k],  e = topk_ids[b,s]
 * FP32 accumulation, bf16 output.  Requirements: hidden % 8 == 0, inter >= 1,
 * 1 <= topk <= 512, x / w_gate_up 16-byte aligned.
 * Replaces warp_decode::launch_moe_gate_up_3d_batched (csrc/moe_gate_up_3d_batched.cu:117-131).
 */
WD_API int wd_moe_gate_up_3d_batched(const void* x, const void* w_gate_up,
                              const int32_t* topk_ids, void* h_out,
                              int B, int E, int topk, int hidden, int inter,
                              uint32_t* status, void* stream);

/*
 * down projection + top-k weighted sum, fused:
 *   y[b, j] = sum_s topk_scale[b,s] * sum_i h[b*topk+s, i] W[e,j,i],  e = topk_ids[b,s]
 * FP32 products and accumulation.  out_fp32 = 0 writes bf16, 1 writes fp32
 * (un-rounded tensor-parallel partial sums).  Requirements: inter % 8 == 0,
 * 1 <= topk <= 512, h / w_down 16-byte aligned.
 * With WARP_DECODE_PDL=1 the launch may start early behind a directly
 * preceding wd_moe_gate_up_3d_batched on the same stream (programmatic
 * dependent launch) and prefetch w_down rows; it reads h and topk_scale only
 * after the preceding kernel has finished, and re-checks topk_ids then.
 * Replaces warp_decode::launch_moe_down_3d_batched (csrc/moe_down_3d_batched.cu:124-141).
 */
WD_API int wd_moe_down_3d_batched(const void* h, const void* w_down,
                           const int32_t* topk_ids, const float* topk_scale,
                           void* y_out, int out_fp32,
                           int B, int E, int topk, int hidden, int inter,
                           uint32_t* status, void* stream);

/*
 * MXFP8-weight variants (no counterpart in the reference).  Activations stay
 * bf16; weights are dequantised in registers (e4m3 * 2^(s-127)) and the dot
 * products accumulate in FP32.  Extra requirements: hidden % 32 == 0
 * (gate_up) / inter % 32 == 0 (down), and the scale tensor's byte size a
 * multiple of 16.
 */
WD_API int wd_moe_gate_up_3d_batched_mxfp8(const void* x, const uint8_t* w_q, const uint8_t* w_scale,
                                    const int32_t* topk_ids, void* h_out,
                                    int B, int E, int topk, int hidden, int inter,
                                    uint32_t* status, void* stream);

WD_API int wd_moe_down_3d_batched_mxfp8(const void* h, const uint8_t* w_q, const uint8_t* w_scale,
                                 const int32_t* topk_ids, const float* topk_scale,
                                 void* y_out, int out_fp32,
                                 int B, int E, int topk, int hidden, int inter,
                                 uint32_t* status, void* stream);

/*
 * Read (and optionally clear) the library-owned status word of the current
 * CUDA device.  Synchronous: it waits for work already queued on the device.
 */
WD_API int wd_status_read(uint32_t* value, int clear);

/*
 * Number of kernels this library has enqueued so far in this process, over
 * all devices and threads.  Counted on the host when a launch is accepted, so
 * a CUDA-graph capture counts the launches it records and a replay counts
 * none; calls rejected by argument checks count none.  No counterpart in the
 * reference (a benchmark reads it around one captured call to report how
 * many kernels the call runs).
 */
WD_API unsigned long long wd_launch_count(void);

/*
 * Choose the kernel behind wd_moe_gate_up_3d_batched (bf16 weights), for all
 * later calls in this process: 0 = automatic (tcgen05 tensor-core kernel from
 * 16 tokens per call, SIMT kernel below), 1 = SIMT kernel only, 2 = tensor-
 * core kernel wherever it applies (E <= 1024).  Both give
 * the same result within bf16 rounding of the FP32 sums.  The environment
 * variable WARP_DECODE_GATE_UP=simt|tc sets the initial choice.  No
 * counterpart in the reference (it has one kernel per op).
 */
WD_API int wd_set_gate_up_path(int path);

/*
 * The same choice for wd_moe_down_3d_batched (bf16 weights): 0 = automatic
 * (tcgen05 kernel from 2 tokens per call), 1 = SIMT kernel only, 2 = tensor-
 * core kernel wherever it applies (inter <= 2048, E <= 1024, hidden <= 128 x
 * the SM count).  WARP_DECODE_DOWN=simt|tc sets the initial choice.  No
 * counterpart in the reference.
 */
WD_API int wd_set_down_path(int path);

/*
 * The whole FFN in one call: gate_up + silu*up, then down + top-k weighted
 * sum (no counterpart in the reference, whose callers make the two calls
 * above back to back: benchmark/bench.py:205,254-255):
 *   h_buf = moe_gate_up(x, w_gate_up, topk_ids)          [B*topk, inter] bf16
 *   y_out = moe_down(h_buf, w_down, topk_ids, topk_scale) [B, hidden] bf16 (fp32 if out_fp32)
 * Same arithmetic and tolerances as the two entry points.  For small calls
 * (automatic choice: B*topk <= 32; forced single launch: <= 64) with x, h of
 * the call fitting in shared memory (E <= 1024 when B*topk > 1) it is ONE
 * cooperative launch of one CTA per SM (SIMT): the down weights stream while
 * gate_up still computes, and a grid barrier orders h.  For larger calls
 * (automatic choice: B*topk >= 65, B <= 64, inter <= 256 and at least 120
 * CTAs of row-tile clusters, e.g. hidden 4096; forced: inter <= 2048) it is
 * ONE cooperative launch on the tensor cores: the bodies of the two tcgen05
 * kernels one after the other on the down kernel's clusters, the routing
 * computed once, each CTA streaming its first down weights as soon as its
 * gate_up items are done, and a grid barrier before h is read.  Otherwise it
 * runs the two kernels of wd_moe_gate_up_3d_batched and
 * wd_moe_down_3d_batched.  Requirements: hidden % 8 == 0, inter % 8 == 0, x,
 * the weights and h_buf 16-byte aligned.
 * sync: 8 bytes of device memory (8-byte aligned; a 64-bit grid-barrier
 * counter), zero before their first use; each single-launch call adds 4096 in
 * total, whatever its grid, and needs nothing else reset.  The counter belongs to
 * one device.  NULL selects a counter owned by the library (one per device).
 * Calls that share a counter must not run at the same time (issue them on one
 * stream, or order them with events); give each concurrently used stream its
 * own.  Every CTA of a call adds its share before it waits, also in a call
 * that ends in WD_STATUS_WAIT_TIMEOUT, so between calls the counter stays a
 * multiple of 4096 and is never reset.
 * Call once per device before capturing it in a CUDA graph (one-time device
 * setup).
 */
WD_API int wd_moe_ffn_3d_batched(const void* x, const void* w_gate_up, const void* w_down,
                                 const int32_t* topk_ids, const float* topk_scale, void* h_buf,
                                 uint32_t* sync, void* y_out, int out_fp32, int B, int E,
                                 int topk, int hidden, int inter, uint32_t* status, void* stream);

/*
 * wd_moe_ffn_3d_batched without h_buf and sync: allocates nothing.  No
 * counterpart in the reference.  h and the grid-barrier counter live in a
 * file-scope static device array of the library (256 B + 128 KiB per
 * device); calls with B*topk*inter*2 > 131072 bytes return
 * WD_ERR_UNSUPPORTED.  The array's counter starts zeroed at module load and,
 * as for wd_moe_ffn_3d_batched, stays a multiple of 4096 after every call (a
 * timed-out one included), so it needs no reset.  The kernels are those of
 * wd_moe_ffn_3d_batched (same choice, same bits).  Every call on a device
 * uses the same array, so calls that overlap in time (other streams) race:
 * serialise them.  The first call on a
 * device looks up the array's address (cudaGetSymbolAddress) and must not be
 * made while that device's stream is being captured.
 */
WD_API int wd_moe_ffn_3d_batched_noalloc(const void* x, const void* w_gate_up, const void* w_down,
                                         const int32_t* topk_ids, const float* topk_scale,
                                         void* y_out, int out_fp32, int B, int E, int topk,
                                         int hidden, int inter, uint32_t* status, void* stream);

/*
 * Router producer (no counterpart in the reference, which takes topk_ids and
 * topk_scale as inputs): from router logits [B, E] (bf16, or fp32 when
 * logits_fp32 != 0) write
 *   topk_ids     [B, topk] int32 = the topk largest logits of each row, in
 *                descending order; equal logits in ascending expert order
 *   topk_weights [B, topk] fp32  = renormalize ? softmax over the selected
 *                logits : softmax over all E logits, at the selected ids
 * NaN logits rank below every number.  1 <= topk <= min(E, 32), E <= 1024.
 * Asynchronous on `stream`; the outputs feed wd_moe_*_3d_batched directly.
 */
WD_API int wd_moe_router_topk(const void* logits, int logits_fp32, int32_t* topk_ids,
                              float* topk_weights, int B, int E, int topk, int renormalize,
                              void* stream);

/*
 * Host <-> device transfers of a decode step by the GPU's own loads and
 * stores, in one launch on `stream` (no copy engine): for i < n, bytes[i]
 * bytes from src[i] to dst[i].  No counterpart in the reference, whose API
 * takes device tensors only; this is how a caller holding x / topk_ids /
 * topk_scale in host memory moves them in, and y out, around
 * wd_moe_ffn_3d_batched (the copy engine's fixed start-up cost dominates
 * transfers of a few KB to a few hundred KB).  Each pointer is memory of the
 * current device or page-locked host memory (cudaHostAlloc, or registered
 * with cudaHostRegister); pageable host memory, or another device's memory,
 * is refused with WD_ERR_UNSUPPORTED before anything is launched.  Ranges
 * must not overlap.  1 <= n <= 4 (n = 0 and empty ranges are no-ops); any
 * alignment (16-byte aligned ranges move in 16-byte units).  Asynchronous:
 * the host may read a dst in host memory once the stream has passed the
 * launch (event or stream synchronisation).
 */
WD_API int wd_copy_ranges(const void* const* src, void* const* dst, const size_t* bytes, int n,
                          void* stream);

/*
 * Kernel choice behind wd_moe_ffn_3d_batched for later calls in this process:
 * 0 = automatic (SIMT single launch up to 32 routed slots, the two kernels up
 * to 64, the tensor-core single launch above where it applies), 1 = always
 * the two kernels, 2 = SIMT single launch wherever it applies (up to 64
 * routed slots), 3 = tensor-core single launch wherever it applies (up to 64
 * tokens).  WARP_DECODE_FFN=split|fused|tc sets the initial choice.
 */
WD_API int wd_set_ffn_path(int path);

/*
 * Which kernels wd_moe_ffn_3d_batched (and its _noalloc twin) would run for
 * these sizes on the current device with the current choice: *kind =
 * WD_FFN_KERNELS_SPLIT (gate_up then down), _SIMT_SINGLE (one SIMT launch)
 * or _TC_SINGLE (one tensor-core launch).  Launches nothing.  No counterpart
 * in the reference.
 */
#define WD_FFN_KERNELS_SPLIT 0
#define WD_FFN_KERNELS_SIMT_SINGLE 1
#define WD_FFN_KERNELS_TC_SINGLE 2
WD_API int wd_moe_ffn_3d_batched_kernels(int B, int E, int topk, int hidden, int inter, int* kind);

/*
 * Tensor parallelism over `inter` with the all-reduce fused into down (no
 * counterpart in the reference, which has no multi-GPU path).  One process
 * per GPU; every rank of a group of `world` (2..8) ranks:
 *   1. wd_tp_comm_create(world, rank, max_tokens, hidden, &comm, handle):
 *      allocates this rank's exchange buffer (2 x world x max_tokens x hidden
 *      8-byte packets: FP32 partial + call epoch) and writes its 64-byte CUDA
 *      IPC handle;
 *   2. gathers every rank's handle (e.g. all_gather over the process group)
 *      into an array of world x 64 bytes ordered by rank and calls
 *      wd_tp_comm_open(comm, handles);
 *   3. calls wd_moe_down_3d_batched_allreduce instead of
 *      wd_moe_down_3d_batched + all-reduce: y_out (bf16 [B, hidden]) is the
 *      sum over all ranks, identical on every rank (ranks added in rank
 *      order).  Every rank must make the same sequence of calls (same B,
 *      shapes and order), like a collective, and enter each call within 2 s
 *      of each other.  Peers exchange rows as epoch-tagged packets through
 *      NVLink peer stores (8-byte single-copy-atomic words, no fences, no
 *      flags), one-shot or two-shot (wd_tp_comm_set_exchange); a peer that does not arrive
 *      within 2 s ends the wait with WD_STATUS_WAIT_TIMEOUT (the output is
 *      then zeros), never a hang.  Needs the tensor-core down kernel's shapes
 *      (inter <= 2048, E <= 1024) and B <= max_tokens per call chunk.
 *   4. wd_tp_comm_destroy(comm) after all ranks are done with it.
 */
WD_API int wd_tp_comm_create(int world, int rank, int max_tokens, int hidden, void** comm,
                             void* ipc_handle);
WD_API int wd_tp_comm_open(void* comm, const void* ipc_handles);
WD_API int wd_tp_comm_destroy(void* comm);
/*
 * Exchange shape of later calls on `comm` (no counterpart in the reference):
 * 0 = by size (default: one-shot with two ranks, and while a rank would
 * send at most 16 MiB, B x hidden x 8 x (world - 1) bytes;
 * WARP_DECODE_TP_TWO_SHOT_BYTES moves the threshold), 1 = one-shot (every
 * rank sums every row), 2 = two-shot
 * (row j summed by rank (j / 4) % world, which sends the bf16 result to the
 * others).  Both give the same bits.  Every rank must set the same mode.
 */
WD_API int wd_tp_comm_set_exchange(void* comm, int mode);
WD_API int wd_moe_down_3d_batched_allreduce(const void* h, const void* w_down,
                                            const int32_t* topk_ids, const float* topk_scale,
                                            void* y_out, int B, int E, int topk, int hidden,
                                            int inter, void* comm, uint32_t* status, void* stream);
/*
 * The whole tensor-parallel FFN with the all-reduce fused in (no counterpart
 * in the reference): this rank's gate_up / down shards, then y_out = bf16
 * sum over all ranks (identical bits on every rank).  Where one of the single
 * launches of wd_moe_ffn_3d_batched applies (SIMT: B*topk <= 32
 * automatically; tensor cores: as for wd_moe_ffn_3d_batched; both with B <= the
 * communicator's max_tokens) that one cooperative kernel also does the
 * exchange; otherwise gate_up, then wd_moe_down_3d_batched_allreduce.
 * h_buf / sync as for wd_moe_ffn_3d_batched; collective rules as above.
 */
WD_API int wd_moe_ffn_3d_batched_allreduce(const void* x, const void* w_gate_up,
                                           const void* w_down, const int32_t* topk_ids,
                                           const float* topk_scale, void* h_buf, uint32_t* sync,
                                           void* y_out, int B, int E, int topk, int hidden,
                                           int inter, void* comm, uint32_t* status, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* WARP_DECODE_B200_H_ */
