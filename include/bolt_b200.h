/*
 * bolt_b200.h -- C ABI of libbolt_b200.so, the B200 (sm_100a) implementation of the
 * nemotron_ops weight-streaming decode ops of the ONNX Runtime custom-op domain "bolt".
 *
 * The reference library exposes exactly one symbol, RegisterCustomOps
 * (src/bolt_ops.cu:1593), and performs each op in a Compute body that reads ORT tensors.
 * This header is the plain-pointer layer underneath: every bolt_* entry point below is the
 * body of one reference op -- same inputs in the same order, same element types and
 * layouts, same attribute meaning, same shape checks and error texts -- with the tensors
 * passed as (device pointer, shape array, rank) and the outputs preallocated by the caller
 * in the shapes the reference op would allocate.  The ORT adapter (nemotron_ops_b200/ort/bolt_ort.cc,
 * built when ORT_INCLUDE_DIR is set) registers the reference's op set over these functions.
 *
 * Conventions
 *   - Pointers are device pointers on the current CUDA device; shapes are host arrays.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Work is only enqueued:
 *     no call synchronises, allocates, or frees memory, so every call can be captured in a
 *     CUDA graph.
 *   - Return value: BOLT_OK, or a nonzero code whose message bolt_last_error() returns
 *     (thread-local).  Shape and launch errors return BOLT_FAIL, as the reference's
 *     ComputeV2 maps them to ORT_FAIL (src/bolt_ops.cu:1464-1466).
 *   - dtypes: "bf16" = bfloat16, "u8" = uint8, "f32" = float, "i32" = int32.
 */
#ifndef BOLT_B200_H_
#define BOLT_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define BOLT_API __attribute__((visibility("default")))
#else
#define BOLT_API
#endif

#define BOLT_OK 0
#define BOLT_FAIL 1             /* same value as ORT_FAIL */
#define BOLT_INVALID_ARGUMENT 2 /* same value as ORT_INVALID_ARGUMENT */

/* Message of the last failing call on this thread ("" if none). */
BOLT_API const char* bolt_last_error(void);

/* ABI version of this header (major * 100 + minor). */
BOLT_API int bolt_abi_version(void);

/*
 * Launch options shared by all ops (process-wide; also read once from the environment
 * variables BOLT_PDL, BOLT_EARLY_WEIGHTS and BOLT_SMEM_BUDGET).
 *   pdl            1 (default): launch the first kernel of an op with programmatic dependent
 *                  launch, so it is scheduled while the previous kernel of the stream drains
 *                  (it still waits for that kernel before touching activations, weights or
 *                  outputs, so results do not change; a preceding kernel that does not trigger
 *                  its dependents early simply completes first).  0: ordinary launches.
 *   early_weights  1: with pdl, stream weights before that wait.  Only valid when the
 *                  kernel immediately preceding an op on the stream does not write the op's
 *                  weights or scales (true for inference graphs with constant weights).
 *                  Default 0.
 *   smem_budget    shared-memory bytes per CTA for staged weights (0 = default).
 * No counterpart in the reference (it has debug knobs BOLT_GEMV_CFG / BOLT_MOE_CFG only).
 */
BOLT_API int bolt_set_launch_options(int pdl, int early_weights, int64_t smem_budget);

/*
 * Reads and clears the device status word of the current device (synchronises the device).
 * Nonzero bits mean a kernel gave up a bounded wait (2 s) and returned without finishing
 * (bits 0-2, 4); bit 3 means a MoE expert id outside [0, E) was skipped; bit 5 means a
 * kernel found its shared-memory carve-out misaligned and returned without computing; bit 6
 * means a MambaVerify `sel` row lay outside its state buffers and nothing was written.
 * No counterpart in the reference.
 */
BOLT_API int bolt_get_device_status(unsigned* status);

/*
 * Nvfp4Gemv (replaces Nvfp4GemvState::ComputeV2, src/bolt_ops.cu:1259-1306; op signature
 * :1565-1574).  y = bf16(g * x @ W^T), W = e2m1 * e4m3 block-16 scale.
 *   x        bf16 [..., K]  (R = numel / K rows, 1 <= R <= 8)
 *   w        u8   [N, K/2]  two e2m1 codes per byte, low nibble first
 *   w_scale  u8   [N, K/16] e4m3 bytes
 *   g        f32  [1]       global scale (device)
 *   y        bf16 [..., N]  (x's shape with the last dim replaced by N)
 * Requires K % 1024 == 0.  (The reference's R = 1 kernel also requires K in {4096, 8192};
 * this implementation does not.)
 */
BOLT_API int bolt_nvfp4_gemv(const void* x, const int64_t* x_shape, int x_rank, const void* w, const int64_t* w_shape,
                    int w_rank, const void* w_scale, const void* g, void* y, void* stream);

/*
 * Q8Gemv (replaces QGemvState<8>::ComputeV2, src/bolt_ops.cu:1429-1468; op :1576-1582).
 *   x       bf16 [..., K], 1 <= R <= 8
 *   B       u8   [N, K/32, 32]  q + 128
 *   scales  bf16 [N, K/32]
 *   y       bf16 [..., N]
 * R = 1 (or K % 64 != 0): exact fp32 weights (q - 128) * s; 2 <= R <= 8: bf16((q - 128) * s).
 */
BOLT_API int bolt_q8_gemv(const void* x, const int64_t* x_shape, int x_rank, const void* B, const int64_t* B_shape, int B_rank,
                 const void* scales, void* y, void* stream);

/*
 * Q4Gemv (replaces QGemvState<4>::ComputeV2, src/bolt_ops.cu:1429-1468; op :1583-1589).
 *   iq2 = 0: B u8 [N, K/32, 16] int4 (zero point 8, low nibble first), scales bf16 [N, K/32]
 *   iq2 = 1: B as iq2 = 0 holding IQ2_XXS LUT codes (mag idx + 4 * neg); 2 <= R <= 8, K % 128 == 0
 *   iq2 = 2: B u8 [N, K/32, 8] native IQ2_XXS records, scales = fp16 bits [N, K/256] in a
 *            bf16-typed tensor; 1 <= R <= 8, K % 256 == 0
 * (The reference's R = 1 int path also limits K <= 6144; this implementation does not.)
 */
BOLT_API int bolt_q4_gemv(const void* x, const int64_t* x_shape, int x_rank, const void* B, const int64_t* B_shape, int B_rank,
                 const void* scales, int64_t iq2, void* y, void* stream);

/*
 * MoeRoute (replaces MoeRouteState::ComputeV2, src/bolt_ops.cu:443-472; op :1521-1530).
 *   x       bf16 [R, K], K % 256 == 0
 *   gate_w  bf16 [E, K], E <= 512
 *   bias    f32  [E]
 *   topk (attribute, <= 32), scale (attribute)
 *   idx     i32  [R, topk]  selection order (bias-corrected score, ties to the lower id)
 *   w       f32  [R, topk]  score / (sum of selected scores + 1e-20) * scale
 *   scores  f32  [R, E]     sigmoid(x @ gate_w^T)
 */
BOLT_API int bolt_moe_route(const void* x, const int64_t* x_shape, int x_rank, const void* gate_w, const int64_t* gw_shape,
                   int gw_rank, const void* bias, int64_t topk, float scale, void* idx, void* w, void* scores,
                   void* stream);

/*
 * MoeDecode (replaces MoeDecodeState::ComputeV2, src/bolt_ops.cu:589-619; op :1531-1544).
 *   z      bf16 [R, 1024]
 *   idx    i32  [R, topk]     expert ids (ids outside [0, E) contribute nothing)
 *   w      f32  [R, topk]
 *   fc1_w  u8   [E, I, 512]   int4, zero point 8;   fc1_s bf16 [E, I, 32]
 *   fc2_w  u8   [E, 1024, I/2];                     fc2_s bf16 [E, 1024, I/32]
 *   out    bf16 [R, 1024];  h bf16 [R*topk, I];  part f32 [R*topk, 1024]
 * Exact fp32 weights.  Requires I % 32 == 0 and R * topk <= 128.
 */
BOLT_API int bolt_moe_decode(const void* z, const int64_t* z_shape, int z_rank, const void* idx, const void* w,
                    const void* fc1_w, const int64_t* fc1_w_shape, int fc1_w_rank, const void* fc1_s, const void* fc2_w,
                    const void* fc2_s, int64_t topk, void* out, void* h, void* part, void* stream);

/*
 * MoeVerify (replaces MoeVerifyState::ComputeV2, src/bolt_ops.cu:1178-1257; op :1545-1557).
 * Inputs as MoeDecode; iq2 = 1: LUT codes in the int4 layout; iq2 = 2: native records
 * fc1_w [E, I, 32, 8] / fc1_s fp16 bits [E, I, 4], fc2_w [E, 1024, I/32, 8] / fc2_s
 * [E, 1024, I/256].  Outputs out, h, part as MoeDecode plus
 *   meta   i32 [1 + P + 8P]   [0] = U unique experts, [1..U] their ids in first-occurrence
 *          order ([U+1..P] = -1), [1 + P + u*8 + row] = pair index (row*topk + k) or -1.
 * Tensor-core weight contract (bf16-rounded weights).  Requires 1 <= R <= 8,
 * R * topk <= 128, I % 64 == 0 (iq2 = 2: I % 256 == 0).
 */
BOLT_API int bolt_moe_verify(const void* z, const int64_t* z_shape, int z_rank, const void* idx, const void* w,
                    const void* fc1_w, const int64_t* fc1_w_shape, int fc1_w_rank, const void* fc1_s, const void* fc2_w,
                    const void* fc2_s, int64_t topk, int64_t iq2, void* out, void* h, void* part, void* meta,
                    void* stream);

/*
 * Expert-sharded MoeVerify step (no counterpart in the reference, which is single-GPU).
 * Computes the op for the experts in [e_begin, e_end) only: `meta` lists the local unique
 * experts, h / part rows of non-local pairs are left untouched, and
 *   out_partial f32 [R, 1024] = sum over local pairs of w * part  (k ascending)
 * is written for the caller to all-reduce (sum) across the shards; `out` (bf16, may be
 * NULL) receives bf16(out_partial).  Only experts in [e_begin, e_end) are read, so a shard may
 * hold just its own experts and pass fc1_w / fc1_s / fc2_w / fc2_s pointers shifted back by
 * e_begin experts, with fc1_w_shape still giving the global expert count.
 */
BOLT_API int bolt_moe_verify_shard(const void* z, const int64_t* z_shape, int z_rank, const void* idx, const void* w,
                          const void* fc1_w, const int64_t* fc1_w_shape, int fc1_w_rank, const void* fc1_s,
                          const void* fc2_w, const void* fc2_s, int64_t topk, int64_t iq2, int64_t e_begin,
                          int64_t e_end, void* out, void* h, void* part, void* meta, void* out_partial, void* stream);

/*
 * Expert-sharded MoeVerify step with the cross-GPU sum built in (no counterpart in the
 * reference, which is single-GPU): bolt_moe_verify_shard, an fp32 all-reduce of the partials and
 * bolt_f32_to_bf16 in one call, with no NCCL.  The last kernel writes this rank's partial into
 * its peer-visible buffer, exchanges flags with the other ranks over NVLink peer memory and adds
 * all ranks' partials in rank order, so `out` bf16 [R, 1024] holds identical bits on every
 * rank.  Every rank of the group must make the same sequence of calls.
 *   peer_bufs   device array [world] of float*: every rank's peer-visible buffer of
 *               2 * half_floats floats (half_floats >= R * 1024) followed by 16 * world uint32
 *               flag words that are zero before the first call
 *   counters    this rank's 16 uint32 call counters (device memory, zero before the first call)
 * Other arguments as bolt_moe_verify_shard (h, part, meta are scratch outputs).  A rank whose
 * peers do not arrive within 2 s stops waiting, leaves `out` unwritten and sets bit 4 of the
 * device status word.
 */
BOLT_API int bolt_moe_verify_shard_allreduce(const void* z, const int64_t* z_shape, int z_rank, const void* idx,
                                             const void* w, const void* fc1_w, const int64_t* fc1_w_shape,
                                             int fc1_w_rank, const void* fc1_s, const void* fc2_w, const void* fc2_s,
                                             int64_t topk, int64_t iq2, int64_t e_begin, int64_t e_end, void* h,
                                             void* part, void* meta, const void* peer_bufs, void* counters,
                                             int64_t half_floats, int64_t rank, int64_t world, void* out,
                                             void* stream);

/*
 * Expert-sharded MoeDecode step (no counterpart in the reference).  As bolt_moe_verify_shard:
 * only pairs whose expert is in [e_begin, e_end) are computed (h / part rows of the other pairs
 * are left untouched), out_partial f32 [R, 1024] receives their weighted sum for the caller to
 * all-reduce, and `out` (bf16, may be NULL) receives bf16(out_partial).  Exact fp32 weights.
 * Requires I % 256 == 0; the weight pointers may be shifted back by e_begin experts as for
 * bolt_moe_verify_shard.
 */
BOLT_API int bolt_moe_decode_shard(const void* z, const int64_t* z_shape, int z_rank, const void* idx, const void* w,
                          const void* fc1_w, const int64_t* fc1_w_shape, int fc1_w_rank, const void* fc1_s,
                          const void* fc2_w, const void* fc2_s, int64_t topk, int64_t e_begin, int64_t e_end,
                          void* out, void* h, void* part, void* out_partial, void* stream);

/*
 * MoeVerify without caller-provided scratch (no counterpart in the reference).  Same inputs,
 * output `out` and contract as bolt_moe_verify; its scratch outputs h, part and meta live in a
 * static 1.5 MiB device buffer inside the library (one per device), so the call allocates
 * nothing.  For callers that cannot allocate device memory at run time (a captured or
 * pre-planned executor, a plugin host that hands out only the op's own outputs) and do not want
 * to carry the three scratch tensors.  Limit: 8192 + R*topk*4096 + R*topk*I*2 bytes (each term
 * rounded up to 256) must fit in 1,572,864 bytes -- R*topk = 64 fits for every I up to 8192,
 * R*topk = 128 for I <= 4064; larger calls fail with a message in bolt_last_error() (use
 * bolt_moe_verify with caller buffers for them).  The first call on a device looks the buffer's
 * address up (cudaGetSymbolAddress) and keeps it for the life of the process; make that call
 * before capturing a stream into a CUDA graph, and do not use the entry point across a
 * cudaDeviceReset of that device.  Nothing has to start at zero: every scratch byte a call reads
 * was written by the same call.  All calls on a device share the buffer, so calls that can
 * overlap in time (different streams or threads) race: the caller must serialise them.
 */
BOLT_API int bolt_moe_verify_noalloc(const void* z, const int64_t* z_shape, int z_rank, const void* idx,
                                     const void* w, const void* fc1_w, const int64_t* fc1_w_shape, int fc1_w_rank,
                                     const void* fc1_s, const void* fc2_w, const void* fc2_s, int64_t topk,
                                     int64_t iq2, void* out, void* stream);

/*
 * MambaStep (replaces MambaStepState::ComputeV2, src/bolt_ops.cu:299-357; kernels :63-297).
 * Attributes heads, head_dim (= 64), d_state (= 128), n_groups, epsilon, time_step_min.
 * di = heads * head_dim, cd = di + 2 * n_groups * d_state.
 *   proj        bf16 [R, di + cd + heads]   rows [gate | xBC | dt], 1 <= R <= 16
 *   conv_state  bf16 [rows, cd, 3];  ssm_state f32 [rows, heads, d_state, head_dim]
 *   conv_w bf16 [cd, 1, 4]; conv_b bf16 [cd]; dt_bias, a_neg, d_skip f32 [heads]; norm_w f32 [di]
 * Outputs: y bf16 [R, di]; conv_state_out / ssm_state_out shaped like the inputs (row 0 = the
 * state after the R tokens, starting from row 0); xbc_act bf16 [R, cd]; ypre f32 [R, di].
 */
BOLT_API int bolt_mamba_step(const void* proj, const int64_t* proj_shape, int proj_rank, const void* conv_state,
                             const int64_t* conv_shape, int conv_rank, const void* ssm_state, const int64_t* ssm_shape,
                             int ssm_rank, const void* conv_w, const void* conv_b, const void* dt_bias,
                             const void* a_neg, const void* d_skip, const void* norm_w, int64_t heads,
                             int64_t head_dim, int64_t d_state, int64_t n_groups, float epsilon, float time_step_min,
                             void* y, void* conv_state_out, void* ssm_state_out, void* xbc_act, void* ypre,
                             void* stream);

/*
 * MambaVerify (the reference's MambaVerifyOp: MambaStepState in verify mode, src/bolt_ops.cu:303,
 * :316-330).  As bolt_mamba_step, plus sel i32 [1] (device): the tokens start from state row
 * *sel and the state after token r is written to row r (needs rows >= R).  A sel outside
 * [0, rows) writes nothing and sets bit 6 of the device status word.
 */
BOLT_API int bolt_mamba_verify(const void* proj, const int64_t* proj_shape, int proj_rank, const void* conv_state,
                               const int64_t* conv_shape, int conv_rank, const void* ssm_state,
                               const int64_t* ssm_shape, int ssm_rank, const void* conv_w, const void* conv_b,
                               const void* dt_bias, const void* a_neg, const void* d_skip, const void* norm_w,
                               const void* sel, int64_t heads, int64_t head_dim, int64_t d_state, int64_t n_groups,
                               float epsilon, float time_step_min, void* y, void* conv_state_out,
                               void* ssm_state_out, void* xbc_act, void* ypre, void* stream);

/*
 * Relu2 (replaces Relu2State::ComputeV2, src/bolt_ops.cu:630-646; kernel :624-629).
 *   x bf16 of any shape (x_shape[x_rank]) -> y bf16 of the same shape,
 *   y = bf16(max(x, 0)^2) with the square in fp32 (a NaN input gives 0, as fmaxf there).
 */
BOLT_API int bolt_relu2(const void* x, const int64_t* x_shape, int x_rank, void* y, void* stream);

/*
 * out[i] = bf16(in[i]) for n f32 values (the cast after the shard all-reduce).
 */
BOLT_API int bolt_f32_to_bf16(const void* in, void* out, int64_t n, void* stream);

/*
 * Stream-ordered copy of `bytes` bytes between host and device memory, either direction (one
 * cudaMemcpyAsync with the direction taken from the pointers; pinned host memory makes it
 * asynchronous).  No reference counterpart: the copy a host caller (ORT, a C or Go binding)
 * issues around an op, exposed so that bindings without a CUDA runtime of their own can stage
 * HOST buffers through this library.
 */
BOLT_API int bolt_memcpy_async(void* dst, const void* src, int64_t bytes, void* stream);

/*
 * Debug / contract check: dequantise N weight rows of K values into f32 [N, K] with the
 * kernels' own decoders.  fmt: 0 = Q8, 1 = Q4 int4, 2 = NVFP4 (e2m1 * e4m3, no global
 * scale), 3 = IQ2 LUT codes, 4 = native IQ2_XXS.  exact = 1 (Q8 / Q4 only) gives the
 * R = 1 contract (q - zp) * s; exact = 0 the tensor-core contract.  Scales as in the ops.
 * No counterpart in the reference.
 */
BOLT_API int bolt_dequant(int fmt, int exact, const void* w, const void* scales, int64_t N, int64_t K, void* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BOLT_B200_H_ */
