/*
 * ats_b200 -- C ABI of the B200 (sm_100a) kernels for the ats-v2 hot path:
 * RMSNorm, rotary embedding and the MoE layer (router, permutation, grouped
 * SwiGLU experts, combine), forward and backward.
 *
 * Conventions
 *   - Every function returns an int status: ATS_OK (0) or a negative ATS_E*
 *     code; ats_last_error_message() gives the detail for this host thread.
 *   - All tensor pointers are device pointers.  The caller allocates every
 *     output and workspace buffer (sizes from the *_workspace_bytes queries);
 *     the library allocates nothing, frees nothing and never synchronises.
 *   - `stream` is a cudaStream_t passed as void*; NULL is the legacy stream.
 *     All work is enqueued on it; calls are re-entrant.
 *   - Arguments are validated on the host before any launch; a bad argument
 *     returns ATS_EBADARG and launches nothing.
 *   - Shapes follow the reference: rows x hidden for norms, [B,H,S,D] views for
 *     RoPE (strides in elements, last dim contiguous), [T,E] router logits.
 *
 * Each entry point names the reference interface (file:line within the
 * ats-v2 project) whose computation it performs.
 */
#ifndef ATS_B200_H
#define ATS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ATS_OK 0
#define ATS_EBADARG (-1)      /* invalid shape, stride, dtype or pointer */
#define ATS_EUNSUPPORTED (-2) /* valid request this build does not implement */
#define ATS_ECUDA (-3)        /* a CUDA launch or runtime call failed */
#define ATS_ETIMEOUT (-4)     /* a bounded device-side wait gave up */

#define ATS_ABI_VERSION 1

#if defined(__GNUC__)
#define ATS_API __attribute__((visibility("default")))
#else
#define ATS_API
#endif

typedef enum ats_dtype { ATS_F32 = 0, ATS_BF16 = 1 } ats_dtype;

ATS_API int ats_abi_version(void);
ATS_API const char* ats_strerror(int status);
ATS_API const char* ats_last_error_message(void);
/* Number of kernels this library has launched in this process (all devices,
 * all threads); a benchmark reads it before and after a timed region. */
ATS_API uint64_t ats_kernel_launches(void);

/* Cap on the CTAs (one per SM) that the persistent tensor-core GEMMs launch
 * with, for launches made later by the calling host thread; 0 (the default)
 * means every SM.  A caller that overlaps a collective on another stream with
 * the expert GEMMs leaves SMs free for it: a GEMM CTA occupies a whole SM, so
 * a collective launched beside a full-width GEMM would wait for its end.
 * No reference counterpart (DeepSpeed's all-to-all does not overlap). */
ATS_API int ats_set_gemm_sm_limit(int sms);
ATS_API int ats_gemm_sm_limit(void);

/* Tile shape of the tensor-core expert, dense-FFN and MLA GEMMs, process-wide:
 * nonzero runs 256-row tiles on pairs of CTAs on two SMs (tcgen05 cta_group::2,
 * each SM loading half of the B tile), zero (the default) runs 128-row tiles on
 * single CTAs.  Both give identical results; a GEMM call reads the setting
 * once.  ats_gemm_pairs returns it.  No reference counterpart. */
ATS_API int ats_set_gemm_pairs(int enable);
ATS_API int ats_gemm_pairs(void);

/* Status of the bounded device waits on the current device: ATS_OK when no
 * wait of a tensor-core GEMM or an RMSNorm ring kernel has given up since the
 * last call, else ATS_ETIMEOUT with the first wait's code in *status; then
 * ATS_EBADARG when a device-driven exchange kernel (ats_moe_ep_push/pull/
 * zero_padding) skipped a row that fell outside its buffer.  Reading clears
 * both.  The outputs of a call whose wait gave up are undefined.
 * Synchronous (copies two ints from the device): call it where the host waits
 * for the device anyway.  No reference counterpart (the reference's kernels
 * have no device-side waits). */
ATS_API int ats_device_status(int* status);

/* Budget, in SM clock cycles, of the main-loop waits of the tensor-core GEMMs
 * and the RMSNorm ring kernels launched later on the current device; <= 0
 * restores the default (about 2 s).  Only a test shortens it, to make a wait
 * run out and check the ATS_ETIMEOUT path; the waits that drain a CTA's copies
 * and MMAs in flight before it exits always keep the default budget.
 * Process-wide per device; not for use while other work runs on the device.
 * No reference counterpart. */
ATS_API int ats_set_wait_budget(int64_t cycles);

/* ------------------------------------------------------------------ RMSNorm
 * y = round(x * rsqrt(mean(x^2) + eps) * w), float32 arithmetic, one rounding
 * to x's dtype.  Replaces RMSNorm.forward, ats/model/norm.py:23-31 (F.rms_norm).
 * x, y: rows x hidden with row strides in elements; w: [hidden] in w_dtype.
 * rstd: optional [rows] float32 output (may be NULL). */
ATS_API int ats_rmsnorm_fwd(const void* x, int64_t x_row_stride, ats_dtype x_dtype,
                    const void* w, ats_dtype w_dtype,
                    void* y, int64_t y_row_stride,
                    float* rstd, int64_t rows, int64_t hidden, float eps, void* stream);

/* Backward of ats_rmsnorm_fwd (autograd of ats/model/norm.py:31):
 *   dx = r*dy*w - x*r^3/H*sum(dy*w*x)   (rounded to x dtype)
 *   dw = sum_rows dy*x*r                 (float32 accumulate, rounded to w dtype)
 * rstd is recomputed from x.  Needs ats_rmsnorm_bwd_workspace_bytes() of
 * workspace (per-block dw partial sums, reduced in a fixed order, so dw is
 * deterministic). */
ATS_API size_t ats_rmsnorm_bwd_workspace_bytes(int64_t rows, int64_t hidden);
ATS_API int ats_rmsnorm_bwd(const void* dy, const void* x, ats_dtype x_dtype,
                    const void* w, ats_dtype w_dtype,
                    void* dx, void* dw,
                    void* workspace, size_t workspace_bytes,
                    int64_t rows, int64_t hidden, float eps, void* stream);

/* Device status of the RMSNorm ring kernels since the library loaded: 0 and
 * ATS_OK when every bounded device-side wait completed, else the wait's code
 * and ATS_ETIMEOUT.  Reading clears the word; the outputs of the call whose
 * wait gave up are undefined.  Synchronous; for diagnostics. */
ATS_API int ats_rmsnorm_status(int* status);

/* Allocation-free variant of ats_rmsnorm_bwd (no counterpart in the
 * reference).  It is meant for callers that cannot allocate device memory
 * around the call: a host runtime that reaches this library through a bare C
 * FFI (cgo, JNI, ctypes) and has no caching allocator of its own, where a
 * cudaMalloc/cudaFree per backward call would stall the device and fragment
 * memory, or a process that runs inside a fixed, pre-reserved memory budget.
 * The caller still passes every input and output; the dw partial sums live
 * in a fixed device array of this library (5 MiB, held by every GPU that
 * loads the library until the process exits).
 *   - hidden must be <= 8192; larger sizes return ATS_EUNSUPPORTED and launch
 *     nothing (use ats_rmsnorm_bwd with a workspace instead).
 *   - The first call on a device looks up that device's address of the array
 *     (cudaGetSymbolAddress with the device current); make that first call
 *     before any stream capture.
 *   - All calls share the one array: calls that overlap on the GPU (different
 *     streams, or other threads, without ordering between them) race on it.
 *     Each call overwrites the part it reads, so no clearing is needed.
 *   - Results equal ats_rmsnorm_bwd's. */
ATS_API int ats_rmsnorm_bwd_noalloc(const void* dy, const void* x, ats_dtype x_dtype,
                            const void* w, ats_dtype w_dtype, void* dx, void* dw,
                            int64_t rows, int64_t hidden, float eps, void* stream);

/* ------------------------------------------------------ RMSNorm + residual
 * out = residual + (x*rsqrt(mean(x^2)+eps)).to(x.dtype) * w with torch type
 * promotion at each step.  Replaces fused_rmsnorm_residual,
 * ats/model/norm_triton.py:101-123 (math of _pytorch_rmsnorm_residual :88-98).
 * x and residual are contiguous rows x hidden of x_dtype; out has dtype
 * promote(x_dtype, w_dtype). */
ATS_API int ats_rmsnorm_residual_fwd(const void* x, const void* residual, ats_dtype x_dtype,
                             const void* w, ats_dtype w_dtype, void* out,
                             int64_t rows, int64_t hidden, float eps, void* stream);

/* Backward: dx (x dtype), dresidual (x dtype), dw (w dtype). dout has dtype
 * promote(x_dtype, w_dtype).  Workspace as ats_rmsnorm_bwd. */
ATS_API int ats_rmsnorm_residual_bwd(const void* dout, const void* x, ats_dtype x_dtype,
                             const void* w, ats_dtype w_dtype,
                             void* dx, void* dresidual, void* dw,
                             void* workspace, size_t workspace_bytes,
                             int64_t rows, int64_t hidden, float eps, void* stream);

/* Residual add fused with the RMSNorm after it, the post-attention step of
 * TransformerBlock.forward (ats/model/transformer.py:208-212: x = residual +
 * attn_out; residual = x; h = post_attention_norm(x)).  sum = round(a + b),
 * the block's next residual, and y = round((sum * rstd(sum)) * w), as
 * ats_rmsnorm_fwd computes it, in one pass over the rows.  a, b, sum, y:
 * rows x hidden contiguous, dtype; w: [hidden] in w_dtype.  Rows of at most
 * 512 16-byte chunks (hidden <= 4096 bf16 or 2048 float32); other shapes return
 * ATS_EUNSUPPORTED. */
ATS_API int ats_add_rmsnorm_fwd(const void* a, const void* b, ats_dtype dtype, const void* w,
                                ats_dtype w_dtype, void* sum, void* y, int64_t rows, int64_t hidden,
                                float eps, void* stream);

/* Backward: dsum = round(round(dnorm) + dsum_in), the gradient of both a and
 * b, where dnorm is the RMSNorm backward of dy and dsum_in (may be NULL: zero)
 * the gradient that reaches sum from its other use (the next residual add) --
 * the order in which autograd sums them; dw (w_dtype) as ats_rmsnorm_bwd, from
 * per-block partial rows in ats_add_rmsnorm_bwd_workspace_bytes() of workspace
 * summed in a fixed order. */
ATS_API size_t ats_add_rmsnorm_bwd_workspace_bytes(int64_t rows, int64_t hidden);
ATS_API int ats_add_rmsnorm_bwd(const void* dy, const void* sum, const void* dsum_in, ats_dtype dtype,
                                const void* w, ats_dtype w_dtype, void* dsum, void* dw, void* workspace,
                                size_t workspace_bytes, int64_t rows, int64_t hidden, float eps,
                                void* stream);

/* ------------------------------------------------------------------- RoPE
 * Rotate-half RoPE on q [B,Hq,S,D] and k [B,Hk,S,D] in one launch:
 *   out = round(round(x*cos) + round(rotate_half(x)*sin)),
 * cos/sin [S,D] tables (row stride cs_row_stride; 0 broadcasts one row to all
 * positions).  backward != 0 applies the
 * adjoint (the gradient w.r.t. x for upstream gradients in *_in).
 * Replaces apply_rotary_pos_emb, ats/model/rope.py:71-87, and fused_apply_rope,
 * ats/model/rope_triton.py:108-128 (k may be NULL, Hk ignored).
 * Strides are in elements for the (b, h, s) dims; D must be contiguous.
 * x_dtype is the dtype of q/k and of cos/sin; outputs have the same dtype. */
ATS_API int ats_rope_apply(const void* q_in, void* q_out, int64_t Hq,
                   const int64_t q_in_strides[3], const int64_t q_out_strides[3],
                   const void* k_in, void* k_out, int64_t Hk,
                   const int64_t k_in_strides[3], const int64_t k_out_strides[3],
                   const void* cos, const void* sin, int64_t cs_row_stride,
                   int64_t B, int64_t S, int64_t D, ats_dtype x_dtype,
                   int backward, void* stream);

/* --------------------------------------------------------------- MoE router
 * Softmax over E experts in float32, top-k (descending; exact ties -> lower
 * expert index), renormalised gates.  Replaces fused_moe_routing,
 * ats/model/moe_triton.py:130-146 (math of _pytorch_moe_routing :121-127) and
 * _PyTorchMoEFallback.compute_routing, ats/model/moe.py:76-90.
 * logits [T,E] float32 contiguous; gates [T,k] float32; idx [T,k] int64;
 * probs: optional [T,E] float32 softmax output (may be NULL). 1 <= k <= E <= 1024, k <= 16. */
ATS_API int ats_moe_topk(const float* logits, int64_t T, int E, int k,
                 float* gates, int64_t* idx, float* probs, void* stream);

/* ------------------------------------------------------- MoE layer (plan)
 * The MoE layer of ats/model/moe.py:92-164 split into device stages that need
 * no host synchronisation.  One workspace (ats_moe_workspace_bytes) carries
 * the routing plan between the stages of a forward and its backward.
 *
 * Permuted ("expert-major") row space, in one of two layouts:
 *   ATS_MOE_PACKED: expert e owns rows [seg_start[e], seg_start[e] + kept_e)
 *     with kept_e = min(count_e, capacity), then zero padding up to a multiple
 *     of 128 rows; the next expert follows (single-GPU layout).
 *   ATS_MOE_SLOTS: expert e owns the fixed rows [e*Cp, e*Cp + kept_e) of a
 *     [E][Cp] buffer, Cp = capacity rounded up to 128, zero padding after the
 *     kept rows -- the send layout of the expert-parallel exchange, where the
 *     buffer reads as [rank][local expert][Cp] (equal all-to-all splits).
 * Tokens inside a segment are in ascending token order (moe.py:109-116).  The
 * number of permuted rows is ats_moe_max_rows(). */
#define ATS_MOE_PACKED 0
#define ATS_MOE_SLOTS 1

ATS_API int64_t ats_moe_max_rows(int64_t T, int E, int k, int64_t capacity, int layout);
ATS_API size_t ats_moe_workspace_bytes(int64_t T, int E, int k, int64_t capacity, int layout);

/* Device status of the MoE stages that ran with this workspace since the last
 * ats_moe_route_plan: writes 0 to *status and returns ATS_OK when every
 * bounded device-side wait completed, else the wait's code and ATS_ETIMEOUT.
 * Synchronous (copies one int from the device); for diagnostics, not the step. */
ATS_API int ats_moe_status(const void* workspace, size_t workspace_bytes, int64_t T, int E, int k,
                   int64_t capacity, int layout, int* status);

/* Copies the plan's segment starts [E+1], the token of every permuted row
 * [max_rows] (-1 = padding) and the kept rows per expert [E] into caller
 * device buffers (any may be NULL), stream-ordered. */
ATS_API int ats_moe_plan_export(const void* workspace, size_t workspace_bytes, int64_t T, int E, int k,
                        int64_t capacity, int layout, int32_t* seg_start, int32_t* row_token,
                        int32_t* kept, void* stream);

/* 1 when the expert GEMMs run this dtype and shape on tcgen05 tensor cores
 * (bf16, hidden and ffn multiples of 128), 0 when on CUDA cores. */
ATS_API int ats_moe_uses_tensor_cores(ats_dtype dtype, int64_t H, int64_t F);

/* Stage 1: route + plan + permutation (moe.py:101-116, :136-162).
 * Writes gates/idx like ats_moe_topk, the workspace plan, and
 *   aux_loss[1]   = E * sum_e mean_t(p[t,e]) * count_e/T * lbw   (float32)
 *   utilization[E] = count_e / max(sum count, 1e-8)               (float32)
 *   counts[E]     = pre-capacity dispatch counts                  (int32)
 * (aux_loss, utilization and counts may be NULL). */
ATS_API int ats_moe_route_plan(const float* logits, int64_t T, int E, int k, int64_t capacity, int layout,
                       float lbw, float* gates, int64_t* idx,
                       float* aux_loss, float* utilization, int32_t* counts,
                       void* workspace, size_t workspace_bytes, void* stream);

/* Stage 2: xp[row] = x[token(row)], zero for padding rows.  x [T,H]; xp [max_rows,H]. */
ATS_API int ats_moe_gather(const void* x, void* xp, ats_dtype dtype, int64_t T, int64_t H,
                   int E, int k, int64_t capacity, int layout,
                   const void* workspace, size_t workspace_bytes, void* stream);

/* Stage 3: the grouped SwiGLU experts (ats/model/ffn.py:37-45 per expert):
 *   h = round(xp Wgu_e^T) [rows,2F] (gate | up), a = round(round(silu(g))*u) [rows,F],
 *   y = round(a Wd_e^T) [rows,H].
 * w_gate_up [E,2F,H] and w_down [E,H,F] contiguous.  bf16 runs on tcgen05
 * tensor cores (float32 accumulate); f32 runs on CUDA cores in float32. */
ATS_API int ats_moe_experts_fwd(const void* xp, const void* w_gate_up, const void* w_down,
                        void* h, void* a, void* y, ats_dtype dtype,
                        int64_t T, int E, int k, int64_t capacity, int layout, int64_t H, int64_t F,
                        const void* workspace, size_t workspace_bytes, void* stream);

/* Stage 4: out[t] = sum over kept (t,e), ascending e, of round(y[row]*gate)
 * accumulated in the token dtype (moe.py:119-122 index_add_).  out [T,H]. */
ATS_API int ats_moe_combine(const void* y, void* out, ats_dtype dtype, int64_t T, int64_t H,
                    int E, int k, int64_t capacity, int layout,
                    const void* workspace, size_t workspace_bytes, void* stream);

/* Backward stage 4: dy[row] = round(dout[token]*gate[row]) (zero on padding),
 * dgate_row[row] = sum_h dout[token,h]*y[row,h] (float32). */
ATS_API int ats_moe_combine_bwd(const void* dout, const void* y, void* dy, float* dgate_row,
                        ats_dtype dtype, int64_t T, int64_t H, int E, int k, int64_t capacity, int layout,
                        const void* workspace, size_t workspace_bytes, void* stream);

/* Backward stage 3: with dh [rows,2F] as caller scratch,
 *   da = round(dy Wd_e); ds = round(da*u); du = round(da*s); dg = round(ds*silu'(g));
 *   dxp = round(dh Wgu_e); dWd_e = round(dy_e^T a_e); dWgu_e = round(dh_e^T xp_e). */
ATS_API int ats_moe_experts_bwd(const void* dy, const void* xp, const void* h, const void* a,
                        const void* w_gate_up, const void* w_down,
                        void* dh, void* dxp, void* dw_gate_up, void* dw_down, ats_dtype dtype,
                        int64_t T, int E, int k, int64_t capacity, int layout, int64_t H, int64_t F,
                        const void* workspace, size_t workspace_bytes, void* stream);

/* Backward stage 2: dx[t] = round(sum over kept rows of token t of dxp[row]),
 * summed in float32 in ascending expert order; zero for tokens with no kept row. */
ATS_API int ats_moe_scatter_grad(const void* dxp, void* dx, ats_dtype dtype, int64_t T, int64_t H,
                         int E, int k, int64_t capacity, int layout,
                         const void* workspace, size_t workspace_bytes, void* stream);

/* Backward stage 1: d(logits) [T,E] float32 from the per-row gate gradients
 * (dgate_row from ats_moe_combine_bwd) through the renormalisation and the
 * softmax, plus the aux-loss term daux * d(aux)/d(probs).  daux is a device
 * pointer to one float32 (the upstream gradient of aux_loss), or NULL for 0. */
ATS_API int ats_moe_route_bwd(const float* logits, const float* gates, const int64_t* idx,
                      const float* dgate_row, const float* daux, float* dlogits,
                      int64_t T, int E, int k, int64_t capacity, int layout, float lbw,
                      const void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------ MoE expert parallelism
 * Expert-parallel MoE (the DeepSpeed MoE path the reference delegates to,
 * ats/model/moe.py:193-214, with ep_size = world size): rank r owns the
 * E_local = E/W experts [r*E_local, (r+1)*E_local).  Each rank plans its own
 * tokens (capacity from its own token count), the host exchanges the row
 * buffers and the kept-row counts with NCCL all-to-all, and the experts run
 * on the received buffer through the segment table built here: the GEMMs
 * compute only the kept rows of each (source, expert) segment (rounded up to
 * 128) and the weight gradients reduce over all W segments of an expert.
 * recv_kept [W*E_local] (device, int32) are the kept rows received from each
 * source for each local expert.  layout says how the received rows lie:
 *   ATS_MOE_SLOTS   [W][E_local][Cp] (equal-split exchange of the sources'
 *                   slot layouts; no host synchronisation);
 *   ATS_MOE_PACKED  the (source, expert) segments back to back, each kept count
 *                   rounded up to 128 (variable-split exchange of the sources'
 *                   packed layouts: only rows the GEMMs read cross the links). */
ATS_API size_t ats_moe_ep_segments_bytes(int W, int E_local);
ATS_API int ats_moe_ep_segments(const int32_t* recv_kept, int W, int E_local, int64_t capacity, int layout,
                        void* seg_workspace, size_t seg_workspace_bytes, void* stream);

/* The grouped SwiGLU experts on the received buffer (rows W*E_local*Cp): as
 * ats_moe_experts_fwd/_bwd with w_gate_up [E_local,2F,H], w_down [E_local,H,F]. */
ATS_API int ats_moe_ep_experts_fwd(const void* xr, const void* w_gate_up, const void* w_down,
                           void* h, void* a, void* y, ats_dtype dtype, int W, int E_local,
                           int64_t capacity, int64_t H, int64_t F,
                           const void* seg_workspace, size_t seg_workspace_bytes, void* stream);
/* ats_moe_ep_experts_fwd on the segments of source ranks [src_lo, src_hi) only
 * (segments are source-major, so they are one range): the rows a rank keeps
 * for its own experts can run while the other ranks' rows are in flight.  The
 * same h, a and y rows as the full call. */
ATS_API int ats_moe_ep_experts_fwd_sources(const void* xr, const void* w_gate_up, const void* w_down,
                           void* h, void* a, void* y, ats_dtype dtype, int W, int E_local,
                           int64_t capacity, int64_t H, int64_t F, const void* seg_workspace,
                           size_t seg_workspace_bytes, int src_lo, int src_hi, void* stream);
ATS_API int ats_moe_ep_experts_bwd(const void* dy, const void* xr, const void* h, const void* a,
                           const void* w_gate_up, const void* w_down,
                           void* dh, void* dxr, void* dw_gate_up, void* dw_down, ats_dtype dtype,
                           int W, int E_local, int64_t capacity, int64_t H, int64_t F,
                           const void* seg_workspace, size_t seg_workspace_bytes, void* stream);

/* Device-driven row exchange of the expert-parallel layer (no reference
 * counterpart: it replaces DeepSpeed's all-to-all dispatch and combine,
 * ats/model/moe.py:207-214, for ranks on one node).  The split sizes never
 * reach the host: every kernel reads the all-gathered counts
 * [W][ats_moe_ep_counts_ints(E)] int32, each rank's row being (kept[E], Cp, R,
 * seg_start[E+1]) from ats_moe_plan_export of its packed-layout plan.  A
 * kept row r of rank `me` in the segment of expert e = d*E_local + p*Ep + j
 * (Ep = E_local/parts) lives in part p of rank d's expert-side buffer at row
 * base + r - seg_start[d*E_local + p*Ep], base = the rounded kept rows the
 * ranks before `me` keep for those experts: the layout ats_moe_ep_segments
 * reads.  peer_bufs [W] (device memory) holds each rank's expert-side buffer
 * (parts x part_rows rows) as an address this process can store to or load
 * from (CUDA IPC mappings; rank `me`'s own buffer as is).  Rows are hidden
 * elements of dtype, a multiple of 16 bytes.  Only kept rows move; the
 * receiver zeroes its padding rows with ats_moe_ep_zero_padding.  No kernel
 * waits on another rank: the caller orders them with collectives (after the
 * counts all-gather; before the expert GEMMs read, or a pull loads, the rows).
 *   push: the kept rows of parts [part_lo, part_hi) into the peers' buffers;
 *         source row r is src[row_token[r]] (tokens) or, with row_token NULL,
 *         src[r] (rows in the packed layout); src has src_rows rows.
 *   pull: the reverse, into dst [dst_rows] in the packed layout. */
ATS_API size_t ats_moe_ep_counts_ints(int E);
ATS_API int ats_moe_ep_push(const void* src, const int32_t* row_token, int64_t src_rows,
                            const int32_t* counts, int W, int me, int E_local, int parts,
                            int part_lo, int part_hi, const uint64_t* peer_bufs, int64_t part_rows,
                            int64_t hidden, ats_dtype dtype, int sms, void* stream);
/* ats_moe_ep_push of only the rows whose expert rank is this rank (to_self
 * nonzero: local stores into its own buffer) or only the others' (zero). */
ATS_API int ats_moe_ep_push_split(const void* src, const int32_t* row_token, int64_t src_rows,
                            const int32_t* counts, int W, int me, int E_local, int parts,
                            int part_lo, int part_hi, const uint64_t* peer_bufs, int64_t part_rows,
                            int64_t hidden, ats_dtype dtype, int to_self, int sms, void* stream);
ATS_API int ats_moe_ep_pull(void* dst, int64_t dst_rows, const int32_t* counts, int W, int me,
                            int E_local, int parts, int part_lo, int part_hi,
                            const uint64_t* peer_bufs, int64_t part_rows, int64_t hidden,
                            ats_dtype dtype, int sms, void* stream);
/* `sms` > 0 sizes a push or pull for that many SMs (it runs beside a GEMM held to the others with
 * ats_set_gemm_sm_limit); 0 sizes it for the whole GPU. */
/* The pull fused with the combine (ats_moe_ep_pull of every part, then
 * ats_moe_combine, bit for bit, in one pass): out[T,hidden] = for each token
 * the gate-weighted sum, ascending expert, of its kept rows' expert outputs,
 * read straight from the expert ranks' buffers (peer_bufs: their mapped
 * addresses, as for ats_moe_ep_pull); each kept row is also stored into the
 * local packed layout ys[ys_rows, hidden] for the backward's
 * ats_moe_combine_bwd.  moe_workspace holds this rank's routing plan (T, k,
 * capacity, W*E_local experts, ATS_MOE_PACKED).  Ordered after the expert
 * GEMMs by the caller's collective, like a pull.  Replaces the reference's
 * index_add_ unpermute (ats/model/moe.py:119-122) across ranks. */
ATS_API int ats_moe_ep_combine(void* ys, int64_t ys_rows, void* out, int64_t T, int k, int64_t capacity,
                               const void* moe_workspace, size_t moe_workspace_bytes, const int32_t* counts,
                               int W, int me, int E_local, int parts, const uint64_t* peer_bufs, int64_t part_rows,
                               int64_t hidden, ats_dtype dtype, void* stream);
ATS_API int ats_moe_ep_zero_padding(void* buf, const int32_t* counts, int W, int me, int E_local,
                                    int parts, int part_lo, int part_hi, int64_t part_rows,
                                    int64_t hidden, ats_dtype dtype, void* stream);

/* ats_moe_ep_experts_bwd in stages: bit 1 the data gradient (dh through the SwiGLU backward, then dxr),
 * bit 2 the weight gradients (dw_gate_up, dw_down; they read dh).  Run data first, then weights, to send
 * dxr on while the weight gradients compute; 3 is ats_moe_ep_experts_bwd. */
ATS_API int ats_moe_ep_experts_bwd_staged(const void* dy, const void* xr, const void* h, const void* a,
                                          const void* w_gate_up, const void* w_down, void* dh, void* dxr,
                                          void* dw_gate_up, void* dw_down, ats_dtype dtype, int W,
                                          int E_local, int64_t capacity, int64_t hidden, int64_t F,
                                          const void* seg_workspace, size_t seg_workspace_bytes,
                                          int stages, void* stream);

/* Device status of the EP expert GEMMs run with this segment workspace (as ats_moe_status). */
ATS_API int ats_moe_ep_status(const void* seg_workspace, size_t seg_workspace_bytes, int W, int E_local,
                      int* status);

/* ------------------------------------------------------------ plain GEMM
 * C[M,N] = A[M,K] . B[N,K]^T in bf16 (float32 accumulation, one rounding) on
 * the expert GEMM kernel as one segment over the rows: the fused MLA KV
 * decompression of ats/model/mla_triton.py:122-151 ((k, v) = (c W_uk^T,
 * c W_uv^T) as one matmul against [W_uk; W_uv]; `_triton_matmul` at :78-104).
 * Needs bf16, M >= 128, N and K multiples of 128 (ats_gemm_supported);
 * A, C, dC, dA are [M, *] row-major, B and dB [N, K].  ats_gemm_bwd writes
 * dA = dC . B and dB = dC^T . A; pass NULL for one to skip it.  The workspace
 * (ats_gemm_workspace_bytes) holds the segment table and the wait status. */
ATS_API int ats_gemm_supported(ats_dtype dtype, int64_t M, int64_t N, int64_t K);
ATS_API size_t ats_gemm_workspace_bytes(void);
ATS_API int ats_gemm_fwd(const void* a, const void* b, void* c, ats_dtype dtype, int64_t M, int64_t N, int64_t K,
                         void* workspace, size_t workspace_bytes, void* stream);
ATS_API int ats_gemm_bwd(const void* dc, const void* a, const void* b, void* da, void* db, ats_dtype dtype, int64_t M,
                         int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* stream);

/* The q/k projection of attention with the rotary embedding in the GEMM's epilogue (row f2 of the hot
 * path: ats/model/attention.py:179-199, q = q_proj(x) viewed [B,S,heads,128], then
 * apply_rotary_pos_emb of ats/model/rope.py:71-87).  out[M,N] (row stride ld_out elements) =
 * rope(x[M,K] . w[N,K]^T), each 128-column head rotated: out[d] = q[d]*cos[d] - q[d+64]*sin[d],
 * out[d+64] = q[d+64]*cos[d+64] + q[d]*sin[d+64], with q the product rounded to bf16 and each product
 * and the sum rounded to bf16 as the reference's bf16 ops round them.  Rows are [batch, seq_len]
 * flattened: row r takes position r % seq_len of cos/sin ([seq_len, 128] bf16, the RotaryEmbedding
 * cache).  bf16 only; M >= 128, N and K multiples of 128.  Workspace as ats_gemm_fwd.  The backward
 * is the RoPE adjoint (ats_rope_apply with backward = 1) followed by ats_gemm_bwd. */
ATS_API int ats_gemm_rope_fwd(const void* x, const void* w, void* out, int64_t ld_out, ats_dtype dtype,
                              int64_t M, int64_t N, int64_t K, const void* cos, const void* sin,
                              int64_t seq_len, void* workspace, size_t workspace_bytes, void* stream);

/* Peer-memory row exchange.  Instead of NCCL all-to-alls, a rank can copy
 * its rows straight into the receive buffers of the experts' ranks with the
 * copy engines (no SMs taken, so the copies run beside the expert GEMMs).
 * ats_ipc_export gives the CUDA IPC handle (ats_ipc_handle_bytes() bytes) of
 * the allocation holding ptr, ptr's offset in it and the allocation's size;
 * a peer process maps it with ats_ipc_open (and ats_ipc_close when done; one
 * open per handle and process).  ats_peer_copies issues n copies
 * dst[i] <- src[i] of bytes[i] bytes on the stream (one cudaMemcpyAsync each;
 * any of them may be a mapped peer address).  The caller orders them against
 * the peers' use of the buffers (a collective before and after).  No
 * reference counterpart: DeepSpeed exchanges with NCCL all-to-alls. */
ATS_API size_t ats_ipc_handle_bytes(void);
ATS_API int ats_ipc_export(const void* ptr, void* handle, uint64_t* offset, uint64_t* alloc_bytes);
ATS_API int ats_ipc_open(const void* handle, void** base);
ATS_API int ats_ipc_close(void* base);
ATS_API int ats_peer_copies(int n, void* const* dst, const void* const* src, const uint64_t* bytes,
                            void* stream);

/* ------------------------------------------------------- dense SwiGLU FFN
 * SwiGLU.forward (ats/model/ffn.py:37-45): y = down(silu(g) * u), [g, u] =
 * chunk(x . w_gate_up^T, 2), for bf16 x [T, hidden], w_gate_up [2F, hidden],
 * w_down [hidden, F], on the same tensor-core GEMMs as the experts (one
 * expert, no routing).  h [R, 2F] and a [R, F] (R = ats_swiglu_rows(T), T
 * rounded up to 128) are saved for the backward; rows past T are zero.
 * Needs T >= 128 and hidden, F multiples of 128 (ats_swiglu_supported). */
ATS_API int ats_swiglu_supported(ats_dtype dtype, int64_t T, int64_t hidden, int64_t F);
ATS_API size_t ats_swiglu_workspace_bytes(void);
ATS_API int64_t ats_swiglu_rows(int64_t T);
ATS_API int ats_swiglu_fwd(const void* x, const void* w_gate_up, const void* w_down, void* h, void* a, void* y,
                   ats_dtype dtype, int64_t T, int64_t hidden, int64_t F, void* workspace,
                   size_t workspace_bytes, void* stream);
/* dy [T, hidden] -> dh [R, 2F] (scratch), dx [T, hidden], dw_gate_up, dw_down (bf16, the weights' layout). */
ATS_API int ats_swiglu_bwd(const void* dy, const void* x, const void* h, const void* a, const void* w_gate_up,
                   const void* w_down, void* dh, void* dx, void* dw_gate_up, void* dw_down,
                   ats_dtype dtype, int64_t T, int64_t hidden, int64_t F, void* workspace,
                   size_t workspace_bytes, void* stream);
ATS_API int ats_swiglu_status(const void* workspace, size_t workspace_bytes, int* status);

/* ------------------------------------------------------- router GEMMs
 * The float32 router of the MoE layer (moe.py:76-90 with the north-star
 * float32 router: logits = x.float() @ w.T) on the tensor cores, for bf16
 * tokens and a float32 weight [E, hidden].  The float32 operands are split
 * into three bf16 parts whose products are exact in the float32 accumulator,
 * so the results are float32 GEMMs up to summation order.  Shapes: bf16
 * tokens, T >= 128, hidden % 128 == 0, 1 <= E <= 64; anything else returns
 * ATS_EUNSUPPORTED (the caller then runs the router with a library GEMM).
 * The workspace is caller-owned (ats_moe_router_workspace_bytes; 0 when the
 * shape is unsupported). */
ATS_API int ats_moe_router_supported(ats_dtype x_dtype, int64_t T, int64_t hidden, int E);
ATS_API size_t ats_moe_router_workspace_bytes(int64_t T, int64_t hidden, int E);

/* logits[T,E] = x[T,hidden] . w[E,hidden]^T (+ bias[E], may be NULL), float32. */
ATS_API int ats_moe_router_fwd(const void* x, const float* w, const float* bias, float* logits,
                       int64_t T, int64_t hidden, int E, void* workspace, size_t workspace_bytes,
                       void* stream);

/* Backward of the router for upstream dlogits [T,E] float32:
 *   dx[T,hidden] (bf16) = bf16(dlogits . w) + bf16(sum of the token's kept
 *     permuted-row gradients dxp, ascending row order) -- the two bf16 token
 *     gradients autograd adds (router input, expert input); with dxp = NULL
 *     only the router's share.  dxp uses the MoE plan in moe_workspace, with
 *     the plan's (T, E, k, capacity, layout); it replaces ats_moe_scatter_grad.
 *   dw[E,hidden] (float32) = dlogits^T . x, summed in a fixed order. */
ATS_API int ats_moe_router_bwd(const float* dlogits, const void* x, const float* w, const void* dxp,
                       const void* moe_workspace, size_t moe_workspace_bytes, int k, int64_t capacity,
                       int layout, void* dx, float* dw, int64_t T, int64_t hidden, int E,
                       void* workspace, size_t workspace_bytes, void* stream);

/* ats_moe_router_bwd in stages, on the same workspace: ATS_ROUTER_BWD_DW splits
 * w and dlogits into their bf16 parts (kept in the workspace) and computes dw;
 * ATS_ROUTER_BWD_DX then computes dx from those parts (x, w and dlogits may be
 * NULL in that call).  The weight gradient needs no expert result, so an
 * expert-parallel backward runs it while the output-gradient rows are in
 * flight.  ATS_ROUTER_BWD_ALL (both) is ats_moe_router_bwd.  No reference
 * counterpart (the reference's router is one nn.Linear). */
#define ATS_ROUTER_BWD_DW 1
#define ATS_ROUTER_BWD_DX 2
#define ATS_ROUTER_BWD_ALL 3
ATS_API int ats_moe_router_bwd_staged(const float* dlogits, const void* x, const float* w, const void* dxp,
                       const void* moe_workspace, size_t moe_workspace_bytes, int k, int64_t capacity,
                       int layout, void* dx, float* dw, int64_t T, int64_t hidden, int E,
                       void* workspace, size_t workspace_bytes, int stages, void* stream);

/* Device status of the router GEMMs run with this workspace (as ats_moe_status). */
ATS_API int ats_moe_router_status(const void* workspace, size_t workspace_bytes, int64_t T, int64_t hidden,
                          int E, int* status);

#ifdef __cplusplus
}
#endif

#endif /* ATS_B200_H */
