/*
 * dsmoe -- B200 (sm_100a) quantized MoE expert layer: C ABI.
 *
 * The drop-in boundary for the reference's MoE hot path. Every entry point takes plain device
 * pointers, sizes and a cudaStream_t (passed as void*), returns an int status (DSMOE_OK = 0,
 * negative on error; dsmoe_last_error() gives the message), launches asynchronously on that
 * stream, and allocates nothing: the caller owns every buffer, including the workspace.
 * This follows the reference's native binding convention (dsv41/ref/fp4lib.py:5-11: raw pointers,
 * integer sizes, caller-owned buffers), with status codes in place of Python-side asserts.
 *
 * Formats:
 *   DSMOE_FMT_FP8  e4m3 weight bytes [out, in] + fp32 scales [ceil(out/128), ceil(in/128)]
 *                  (dsv41/ref/kernel.py:75-78)
 *   DSMOE_FMT_FP4  e2m1 codes [out, in/2], low nibble first + e8m0 scales [out, in/32]
 *                  (dsv41/ref/kernel.py:91-98; dsv41/ref/fp4lib.c:12-30; dsv41/ckpt.py:41-50)
 */
#ifndef DSMOE_H_
#define DSMOE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DSMOE_API __attribute__((visibility("default")))
#else
#define DSMOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define DSMOE_OK 0
#define DSMOE_ERR_ARG (-1)         /* bad shape, null pointer, unsupported combination */
#define DSMOE_ERR_ALIGN (-2)       /* pointer not 16-byte aligned */
#define DSMOE_ERR_CUDA (-3)        /* a CUDA call or launch failed */
#define DSMOE_ERR_WORKSPACE (-4)   /* workspace too small */
#define DSMOE_ERR_TIMEOUT (-5)     /* a bounded device-side wait gave up */
#define DSMOE_ERR_UNSUPPORTED (-6)

#define DSMOE_FMT_FP8 0
#define DSMOE_FMT_FP4 1

#define DSMOE_SCORE_SIGMOID 0
#define DSMOE_SCORE_SQRTSOFTPLUS 1

#define DSMOE_DTYPE_F32 0
#define DSMOE_DTYPE_BF16 1
#define DSMOE_DTYPE_E4M3 2

/* Largest decode batch of dsmoe_moe_decode (tokens per call). */
#define DSMOE_MAX_DECODE_TOKENS 64
/* Tokens per expert slot in a decode step: an expert chosen by more tokens gets more slots,
 * the "virtual bucket" rule of dsv41/tt/moe.py:184-187 with a bucket of 8 rows. */
#define DSMOE_SLOT_TOKENS 8

/* Resident store layouts. */
#define DSMOE_LAYOUT_FRAG 0  /* packed fragment-order tiles, scales co-located (dsmoe_store_pack_expert) */
#define DSMOE_LAYOUT_TC 1    /* checkpoint row-major weights + per-tile scale tables, read by the
                                tensor-core decode path through TMA tensor maps (dsmoe_store_tc_pack_expert) */

/* One expert set of one layer on this GPU, in one of the resident layouts. */
typedef struct dsmoe_store {
  const uint8_t* w13;          /* [n_experts][w13_expert_bytes] */
  const uint8_t* w2;           /* [n_experts][w2_expert_bytes]  */
  long long w13_expert_bytes;  /* dsmoe_store_expert_bytes() / dsmoe_store_tc_expert_bytes() */
  long long w2_expert_bytes;
  int fmt;                     /* DSMOE_FMT_* */
  int n_experts;
  int layout;                  /* DSMOE_LAYOUT_* (0 for a zero-initialised struct) */
  int row0;                    /* DSMOE_LAYOUT_TC: first intermediate row of this GPU's slice */
} dsmoe_store_t;

/* One MoE layer on this GPU: router, routed experts and the shared expert.
 * With tensor parallelism over W GPUs, each GPU holds inter_local = I / W rows of every expert's
 * intermediate dimension (w1/w3 column-parallel, w2 row-parallel; dsv41/tt/moe.py:2-3) and the
 * layer output on each GPU is a partial sum to be all-reduced. */
typedef struct dsmoe_layer {
  int hidden;                  /* H */
  int inter_local;             /* intermediate rows per expert on this GPU */
  int n_experts;               /* routed experts E */
  int topk;                    /* k <= 8 */
  int score_func;              /* DSMOE_SCORE_* */
  float route_scale;
  const float* gate_w;         /* [E, H] fp32 router weight (checkpoint [out, in] layout) */
  const float* gate_bias;      /* [E] fp32, selection-only bias */
  const float* gate_bias_vl;   /* [E] fp32 or NULL: bias for image-span tokens */
  dsmoe_store_t routed;
  dsmoe_store_t shared;        /* one expert */
} dsmoe_layer_t;

DSMOE_API const char* dsmoe_last_error(void);
DSMOE_API int dsmoe_version(void);

/* ---- weight unpack (kernel-surface dequant) ------------------------------------------------ */

/* FP8 block dequant: b [N, K] e4m3, b_s [ceil(N/block), ceil(K/block)] fp32 -> out [N, K].
 * Replaces `_deq_fp8_weight` (dsv41/ref/kernel.py:75-78) and the `weight_dequant` kernel entry
 * point of DeepSeek's inference/kernel.py. out_dtype: DSMOE_DTYPE_F32 or DSMOE_DTYPE_BF16. */
DSMOE_API int dsmoe_fp8_block_dequant(const uint8_t* b, const float* b_s, long long N, long long K, int block,
                            void* out, int out_dtype, void* stream);

/* FP4 dequant: b [N, K/2] packed e2m1, b_s [N, K/32] e8m0 -> out [N, K].
 * Replaces `dequant_fp4_weight` (dsv41/ref/kernel.py:91-98) and `dequant_fp4`
 * (dsv41/ref/fp4lib.c:12-30). */
DSMOE_API int dsmoe_fp4_dequant(const uint8_t* b, const uint8_t* b_s, long long N, long long K,
                      void* out, int out_dtype, void* stream);

/* ---- kernel-surface GEMMs and activation quant ------------------------------------------- */

/* out[M, N] = (a * a_s per 128-K block) @ dequant(b, b_s)^T, rounded to out_dtype.
 * a: [M, K] in a_dtype (F32, BF16 or E4M3), a_s: [M, K/128] fp32 or NULL (all ones).
 * Replaces `fp8_gemm` (dsv41/ref/kernel.py:105-107). */
DSMOE_API int dsmoe_fp8_gemm(const void* a, int a_dtype, const float* a_s, long long M, long long K,
                   const uint8_t* b, const float* b_s, long long N, void* out, int out_dtype,
                   void* stream);

/* Same with FP4 weights b [N, K/2] + e8m0 b_s [N, K/32]. Replaces `fp4_gemm`
 * (dsv41/ref/kernel.py:110-112). */
DSMOE_API int dsmoe_fp4_gemm(const void* a, int a_dtype, const float* a_s, long long M, long long K,
                   const uint8_t* b, const uint8_t* b_s, long long N, void* out, int out_dtype,
                   void* stream);

/* Per-(row, block) e4m3 activation quant: s = amax/448 (or its power-of-2 ceiling when pow2 != 0),
 * q = e4m3(clamp(x / s, +-448)), amax clamped below at 1e-4. Replaces the quantizing branch of
 * `act_quant` (dsv41/ref/kernel.py:44-55). x: [M, K] in x_dtype (F32 or BF16). */
DSMOE_API int dsmoe_act_quant(const void* x, int x_dtype, long long M, long long K, int block, int pow2,
                    uint8_t* q, float* s, void* stream);

/* ---- expert store (one-time repack; replaces the host ExpertStore / tile packer) ---------- */

/* Bytes of one expert's w1|w3 part and w2 part in the packed store. */
DSMOE_API int dsmoe_store_expert_bytes(int fmt, int hidden, int inter_local, long long* w13_bytes,
                             long long* w2_bytes);

/* Repack one expert from checkpoint layout (device memory) into the packed store, keeping
 * intermediate rows [row0, row0 + inter_local) -- this GPU's tensor-parallel slice.
 *   FP8: w1,w3 [I, H] e4m3, s1,s3 fp32 [ceil(I/128), H/128]; w2 [H, I] e4m3, s2 fp32 [H/128, ceil(I/128)]
 *   FP4: w1,w3 [I, H/2] u8, s1,s3 e8m0 [I, H/32];         w2 [H, I/2] u8,  s2 e8m0 [H, I/32]
 * Replaces ExpertStore._pack_one_proj / pack_expert_fp4_shards (dsv41/tt/store.py:66-89;
 * dsv41/ref/fp4lib.c:116-186), which packed Tenstorrent tiles on the host. */
DSMOE_API int dsmoe_store_pack_expert(int fmt, int hidden, int inter, int row0, int inter_local,
                            const uint8_t* w1, const void* s1, const uint8_t* w3, const void* s3,
                            const uint8_t* w2, const void* s2, uint8_t* w13_dst, uint8_t* w2_dst,
                            void* stream);

/* Inverse of dsmoe_store_pack_expert, dequantized to fp32: w1,w3 [inter_local, H], w2 [H, inter_local].
 * Used to prove the packed store is lossless (bit-exact against the reference dequant). */
DSMOE_API int dsmoe_store_unpack_expert(int fmt, int hidden, int inter, int row0, int inter_local,
                              const uint8_t* w13_src, const uint8_t* w2_src, float* w1, float* w3,
                              float* w2, void* stream);

/* Tensor-core store (DSMOE_LAYOUT_TC): the expert's rows [row0, row0 + inter_local) kept in the
 * checkpoint's own row-major order (FP8 bytes / packed FP4 bytes as stored), w2 rows padded to whole
 * 128-K blocks, and the scales rearranged into per-tile tables; the decode kernel's TMA tensor maps
 * tile and swizzle the weights on the fly. Same inputs and slice rules as dsmoe_store_pack_expert
 * (hidden a multiple of 128; row0, inter_local and inter multiples of 32). Replaces the same
 * reference packers (dsv41/tt/store.py:66-89; dsv41/ref/fp4lib.c:116-186). Destinations 1024-byte
 * aligned; expert strides from dsmoe_store_tc_expert_bytes. */
DSMOE_API int dsmoe_store_tc_expert_bytes(int fmt, int hidden, int inter, int row0, int inter_local,
                                          long long* w13_bytes, long long* w2_bytes);
DSMOE_API int dsmoe_store_tc_pack_expert(int fmt, int hidden, int inter, int row0, int inter_local,
                                         const uint8_t* w1, const void* s1, const uint8_t* w3, const void* s3,
                                         const uint8_t* w2, const void* s2, uint8_t* w13_dst, uint8_t* w2_dst,
                                         void* stream);
/* Inverse of dsmoe_store_tc_pack_expert through its scale tables, dequantized to fp32
 * (w1, w3 [inter_local, H], w2 [H, inter_local]): proves the layout lossless. */
DSMOE_API int dsmoe_store_tc_unpack_expert(int fmt, int hidden, int inter, int row0, int inter_local,
                                           const uint8_t* w13_src, const uint8_t* w2_src, float* w1, float* w3,
                                           float* w2, void* stream);

/* ---- router and MoE forward --------------------------------------------------------------- */

/* Workspace bytes for dsmoe_router / dsmoe_moe_decode at batch B. */
DSMOE_API size_t dsmoe_moe_workspace_bytes(const dsmoe_layer_t* layer, int B);

/* On-device router: logits = x @ gate_w^T (fp64 accumulation, rounded to fp32), scores =
 * score_func(logits), top-k of scores + bias (ties -> lower expert index), weights = the unbiased
 * scores at those indices / (sum + 1e-20) * route_scale.
 * Replaces MoE.scores + MoE.pick_from_host (dsv41/tt/moe.py:108-125), which read the scores back
 * to the host every layer. x [B, H] bf16; image_mask [B] u8 or NULL selects gate_bias_vl per token.
 * Outputs: idx [B, k] int64, wt [B, k] fp32, scores [B, E] fp32 (scores may be NULL). */
DSMOE_API int dsmoe_router(const dsmoe_layer_t* layer, const void* x, int B, const uint8_t* image_mask,
                 int64_t* idx, float* wt, float* scores, void* workspace, size_t workspace_bytes,
                 void* stream);

/* dsmoe_router with no caller workspace and no allocation: the scratch is a 1,315,072-byte array in
 * the library's own device image (limits B <= 64, n_experts <= 1024, hidden <= 8192, topk <= 8;
 * larger calls return DSMOE_ERR_ARG). For callers that cannot provide device scratch memory.
 * The first call on a device (with that device current) resolves the array's address and must
 * come before any stream capture; calls on one device must not overlap (they share the array).
 * The resolved address is kept for the life of the process: it is not valid across a
 * cudaDeviceReset or a re-created primary context of that device.
 * Same outputs as dsmoe_router. No counterpart in the reference. */
DSMOE_API int dsmoe_router_noalloc(const dsmoe_layer_t* layer, const void* x, int B, const uint8_t* image_mask,
                                   int64_t* idx, float* wt, float* scores, void* stream);

/* Whole MoE layer for B <= DSMOE_MAX_DECODE_TOKENS tokens: router, routed experts (each weight
 * tile read once per step for all tokens that chose it), shared expert, routing-weighted combine.
 * Replaces MoE.decode / verify_batched (dsv41/tt/moe.py:148-180, 202-241).
 * For B <= 8 (hidden a multiple of 512, <= 1024 experts) the layer runs as one persistent kernel
 * that keeps counters and a grid barrier in the workspace: the workspace must be zero-filled once
 * before its first use (calls leave it reusable), and calls sharing one workspace must not overlap
 * on the GPU. Every device-side wait is bounded; dsmoe_moe_check reports an expired wait. After
 * an expired wait the workspace's status word stays set, and every later persistent call on that
 * workspace writes NaN into y (it never leaves y unwritten) until dsmoe_moe_check resets it.
 * y: [B, H]; y_dtype DSMOE_DTYPE_BF16 (final output) or DSMOE_DTYPE_F32 (this GPU's partial sum,
 * before the all-reduce). idx/wt/scores as in dsmoe_router (each may be NULL). */
DSMOE_API int dsmoe_moe_decode(const dsmoe_layer_t* layer, const void* x, int B, const uint8_t* image_mask,
                     void* y, int y_dtype, int64_t* idx, float* wt, float* scores,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Synchronizes `stream` and reads the status word of the persistent path: DSMOE_OK, or
 * DSMOE_ERR_TIMEOUT when a bounded device-side wait expired in an earlier call (the workspace
 * counters are then reset). Failure detection for the path; no counterpart in the reference. */
DSMOE_API int dsmoe_moe_check(const dsmoe_layer_t* layer, int B, void* workspace, size_t workspace_bytes,
                              void* stream);

/* dsmoe_moe_decode that also records four caller-created CUDA events on the stream: before the
 * router kernels, before the w1|w3 kernel, before the w2 kernel and after it. Same work, same
 * results; used by the benchmark to time each kernel on its own stream (no counterpart in the
 * reference, whose bench times whole traces, bench/bench_layer.py:34-51). On the persistent path
 * the first three events are recorded together before its single kernel. */
DSMOE_API int dsmoe_moe_decode_profiled(const dsmoe_layer_t* layer, const void* x, int B,
                                        const uint8_t* image_mask, void* y, int y_dtype, int64_t* idx,
                                        float* wt, float* scores, void* workspace, size_t workspace_bytes,
                                        void* stream, void* const* events);

/* fp32 [n] -> bf16 [n] (the last step after an fp32 all-reduce of the partial sums). */
DSMOE_API int dsmoe_f32_to_bf16(const float* src, void* dst, long long n, void* stream);

/* One asynchronous copy of n bytes between addresses the device can reach (device memory or
 * page-locked host memory), ordered on the stream. Under CUDA-graph capture it becomes one memcpy
 * node: the traced decode step (the role of DecodeTrace, dsv41/tt/model.py:262-330) copies its
 * tokens in and its outputs out with it. Pageable host memory is rejected during capture. */
DSMOE_API int dsmoe_copy_async(void* dst, const void* src, long long n, void* stream);

/* ---- prefill / batched layer on the 5th-generation tensor cores --------------------------- */

/* Workspace bytes for dsmoe_moe_prefill with P tokens (0 if the layer or P is unsupported). */
DSMOE_API size_t dsmoe_moe_prefill_workspace_bytes(const dsmoe_layer_t* layer, int P);

/* Whole MoE layer for P = 1..4096 tokens with given routing: idx [P, k] int64 and wt [P, k] fp32
 * (from dsmoe_router, or forced), x [P, H] bf16 (16-byte aligned), y [P, H] bf16 or fp32 (this
 * GPU's partial with y_dtype F32). The (token, expert) pairs are grouped by expert (counting sort,
 * chunks of <= 64 tokens), then two grouped GEMMs on tcgen05 with TMEM accumulators: w1|w3 per
 * chunk, SwiGLU, w2 per chunk, and a routing-weighted combine in k order plus the shared expert.
 * FP8 experts use kind::f8f6f4 with their 128 x 128 fp32 scales applied per 128-K block to the
 * accumulator; FP4 experts use kind::mxf8f6f4.block_scale with their e8m0 scales. Requires
 * hidden and inter_local multiples of 128 and P * k <= 8192. Every device wait is bounded;
 * dsmoe_moe_prefill_check reports an expired wait or an out-of-range expert index.
 * Replaces MoE.prefill_batched / _batched (dsv41/tt/moe.py:182-200, 263-288) and MoE.prefill
 * (dsv41/tt/moe.py:290-303). */
DSMOE_API int dsmoe_moe_prefill(const dsmoe_layer_t* layer, const void* x, int P, const int64_t* idx,
                                const float* wt, void* y, int y_dtype, void* workspace, size_t workspace_bytes,
                                void* stream);

/* Synchronizes `stream` and reads the prefill status word: DSMOE_OK, DSMOE_ERR_TIMEOUT (a bounded
 * wait expired) or DSMOE_ERR_ARG (an expert index outside 0..n_experts-1); clears it. */
DSMOE_API int dsmoe_moe_prefill_check(const dsmoe_layer_t* layer, int P, void* workspace, size_t workspace_bytes,
                                      void* stream);

/* ---- all-reduce inside the decode kernel (tensor parallelism over NVLink peers) ----------- */

/* One rank's end of a tensor-parallel group for dsmoe_moe_decode_allreduce: an exchange buffer in
 * this GPU's memory that the other ranks map with CUDA IPC. Replaces the reference's per-layer
 * all_reduce_sum (dsv41/tt/attn.py:19-21, called at dsv41/tt/moe.py:162, 180).
 * Set-up: every rank calls dsmoe_comm_create (with its device current), the ranks exchange the
 * DSMOE_COMM_HANDLE_BYTES-byte handles (any host channel), then every rank calls dsmoe_comm_open
 * with all handles concatenated in rank order. world 2..8; hidden must match the layers'. */
#define DSMOE_COMM_HANDLE_BYTES 64
typedef struct dsmoe_comm dsmoe_comm_t;
DSMOE_API int dsmoe_comm_create(int rank, int world, int hidden, dsmoe_comm_t** comm, void* handle_out);
DSMOE_API int dsmoe_comm_open(dsmoe_comm_t* comm, const void* handles);
/* Synchronizes the device, unmaps the peers' buffers and frees this rank's. */
DSMOE_API int dsmoe_comm_destroy(dsmoe_comm_t* comm);

/* y[b][:] = the sum over the group's ranks of x[b][:] for B = 1..8 rows of `hidden` values (bf16 or
 * fp32 in and out), over the same NVLink peer exchange as dsmoe_moe_decode_allreduce: one launch,
 * the sum in rank order (the same bits on every rank). Replaces the reference's all_reduce_sum of
 * the attention output projection (dsv41/tt/attn.py:19-21, called at attn.py:229, 252). Every rank
 * makes the same sequence of calls on one comm (this and the decode call share its epochs). */
DSMOE_API int dsmoe_allreduce_rows(const dsmoe_comm_t* comm, const void* x, int x_dtype, int B, void* y,
                                   int y_dtype, void* stream);
/* Synchronizes `stream` and reads the comm's status word: DSMOE_OK, or DSMOE_ERR_TIMEOUT when a
 * peer's tile did not arrive within the bound in dsmoe_allreduce_rows (the comm must then be
 * re-created on every rank); clears it. */
DSMOE_API int dsmoe_comm_check(const dsmoe_comm_t* comm, void* stream);

/* 1 when dsmoe_moe_decode_allreduce takes this call (the persistent path: B <= 8 tokens, hidden a
 * multiple of 512, <= 1024 experts, x 16-byte aligned), else 0. */
DSMOE_API int dsmoe_moe_allreduce_supported(const dsmoe_layer_t* layer, const dsmoe_comm_t* comm, const void* x,
                                            int B);

/* dsmoe_moe_decode whose output y is the sum of every rank's partial: each rank's persistent
 * kernel stores its output tiles into the peers' exchange buffers over NVLink and sums the tiles
 * it receives in rank order, so y is bit-identical on every rank and the layer is one launch per
 * rank. All ranks must make the same sequence of calls on one comm (layers may share it); calls on
 * one comm must not overlap. A peer that has not delivered a tile within 5 s sets a status bit
 * that dsmoe_moe_check reports; the comm must then be destroyed and re-created on every rank.
 * Returns DSMOE_ERR_UNSUPPORTED when dsmoe_moe_allreduce_supported is 0 (use dsmoe_moe_decode with
 * y_dtype F32 and a collective library then). */
DSMOE_API int dsmoe_moe_decode_allreduce(const dsmoe_layer_t* layer, const dsmoe_comm_t* comm, const void* x,
                                         int B, const uint8_t* image_mask, void* y, int y_dtype, int64_t* idx,
                                         float* wt, float* scores, void* workspace, size_t workspace_bytes,
                                         void* stream);

#ifdef __cplusplus
}
#endif
#endif /* DSMOE_H_ */
