/*
 * fd_b200.h -- C ABI of the B200 (sm_100a) decode-step kernels.
 *
 * Every entry point takes plain device pointers, element strides, sizes and a
 * cudaStream_t passed as `void*`.  No PyTorch type crosses this boundary.  All
 * launches are asynchronous on the given stream, never synchronise the host and
 * may be captured into a CUDA graph (workspaces are caller-owned and the
 * kernels leave them ready for the next launch).
 *
 * The entry points replace the launcher layer of the reference package
 * fused_decode (src/fused_decode/kernels.py).  Each declaration names the
 * reference function it stands in for.  Argument meaning follows the reference:
 * strides are in ELEMENTS, rows are described by the reference's RowLayout
 * (up to three leading dimensions plus the last-dimension stride).
 *
 * Return value: FD_OK (0) or an fd_status code; fd_status_string() names it.
 */
#ifndef FD_B200_H
#define FD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types.  Activations are f16/bf16; norm weights, RoPE angles, bias and
 * row_add may also be f32 (reference ops.py:20-21, 126, 196, 248). */
typedef enum {
  FD_F16 = 0,
  FD_BF16 = 1,
  FD_F32 = 2
} fd_dtype;

typedef enum {
  FD_OK = 0,
  FD_ERR_ARG = 1,         /* bad pointer, size, stride or dtype combination */
  FD_ERR_LAUNCH = 2,      /* the CUDA launch itself failed */
  FD_ERR_WORKSPACE = 3,   /* workspace missing or smaller than required */
  FD_ERR_UNSUPPORTED = 4, /* shape outside what the entry point covers */
  FD_ERR_DEVICE = 5       /* device query failed */
} fd_status;

/* GEMV kinds, as the reference's `kind=` strings (kernels.py:581-586). */
typedef enum {
  FD_KIND_DOT = 0,  /* tensor-core path (reference "dot") */
  FD_KIND_SIMT = 1  /* CUDA-core fp32 FMA path (reference "simt") */
} fd_kind;

/* A batch of rows of length n.  Row r = (ia, ib, ic) with r = (ia*b + ib)*c + ic
 * starts at ptr + ia*sa + ib*sb + ic*sc; element j of the row is at +j*col.
 * Mirrors RowLayout / row_layout / _row_base (reference kernels.py:26-88). */
typedef struct {
  void* ptr;
  int32_t dtype; /* fd_dtype */
  int32_t _pad;
  int64_t a, b, c;
  int64_t sa, sb, sc;
  int64_t col;
  int64_t n;
} fd_rows;

const char* fd_status_string(int status);

/* Number of SMs of the current device, as the kernels size their grids. */
int fd_device_sm_count(void);

/* RMSNorm and fused add+RMSNorm over the last dimension.
 *   s = x (+ residual)             (fp32)
 *   residual_out = round(s)        (if residual_out != NULL; may alias residual)
 *   out = round(s * rsqrt(mean(s*s) + eps) * weight)
 * residual / residual_out may be NULL.  weight is [n] with element stride
 * w_stride and dtype w_dtype (f16, bf16 or f32).
 * Replaces rms_out (reference kernels.py:343-414). */
int fd_rms_out(const fd_rows* x, const fd_rows* residual, const void* weight,
               int32_t w_dtype, int64_t w_stride, const fd_rows* out,
               const fd_rows* residual_out, float eps, void* stream);

/* out = round(silu(gate) * up), fp32 math, stable sigmoid.
 * Replaces swiglu_out (reference kernels.py:456-487). */
int fd_swiglu_out(const fd_rows* gate, const fd_rows* up, const fd_rows* out,
                  void* stream);

/* Rotate-half RoPE.  cos/sin are already broadcast to x's row grid (stride 0
 * where they broadcast) and may be f16, bf16 or f32 independently of x.
 *   out[:h] = x1*c1 - x2*s1,  out[h:] = x2*c2 + x1*s2
 * Replaces rope_out (reference kernels.py:541-578). */
int fd_rope_out(const fd_rows* x, const fd_rows* cos, const fd_rows* sin,
                const fd_rows* out, void* stream);

/* Workspace bytes fd_linear_out needs for this shape.  The workspace must be
 * zero-filled once when first allocated; every launch leaves its counters at
 * zero again, so one buffer serves every later launch on the same stream
 * (launches that share a workspace must not overlap in time). */
size_t fd_linear_workspace_bytes(int32_t m, int64_t n, int64_t k);

/* Byte offset, inside any workspace above, of a 32-bit status word the
 * kernels OR error bits into (1: a consumer's shared-memory pipeline wait
 * expired, 2: a producer's wait expired, 8: a tensor-parallel exchange wait
 * expired, 16: a grid-wide barrier wait of the persistent MLP stack expired).  Zero means no error.  After a non-zero
 * status the outputs of that launch are invalid and the workspace must be
 * zero-filled again before reuse. */
size_t fd_workspace_status_offset(void);

/* y[m, n] = round(sum_k x[m, k] * w[n, k] + bias[n] + row_add[m, n]) for
 * 1 <= m <= 16, fp32 accumulation.  bias (dtype = x dtype or f32) and row_add
 * (f16, bf16 or f32; stride 0 where it broadcasts) may be NULL.  dtype is the
 * activation dtype shared by x, w and y.  kind is an fd_kind.
 * Replaces linear_out (reference kernels.py:741-830). */
int fd_linear_out(const void* x, int64_t sxm, int64_t sxk,
                  const void* w, int64_t swn, int64_t swk,
                  const void* bias, int32_t bias_dtype, int64_t sbias,
                  const void* row_add, int32_t ra_dtype, int64_t srm, int64_t srn,
                  void* y, int64_t sym, int64_t syn,
                  int32_t dtype, int32_t m, int64_t n, int64_t k, int32_t kind,
                  void* workspace, size_t workspace_bytes, void* stream);

/* fd_linear_out without a workspace argument.  No counterpart in the
 * reference (its launchers allocate through PyTorch).  For callers that have
 * no device memory to hand over -- a host without an allocator of its own, or
 * one whose memory plan forbids device allocation after start-up -- the
 * split-K scratch lives in the library's static device memory: at most
 * fd_linear_noalloc_scratch_bytes() (6 MiB) per device.  Nothing is allocated.
 *   - The first call on a device looks up that device's scratch address
 *     (set-up, done once per device; make it before any stream capture).
 *   - The scratch starts at zero when the library is loaded on a device, and
 *     every completed launch leaves its counters at zero again; after a
 *     launch whose wait expired, fd_linear_noalloc_reset() below restores it.
 *   - All calls on one device share the one scratch: calls that overlap in
 *     time (concurrent streams, threads) race; serialise them.
 *   - Returns FD_ERR_WORKSPACE when the device needs more scratch than the
 *     built-in size (fd_linear_workspace_bytes() above it, i.e. a GPU with more
 *     than 183 SMs); otherwise the return values of fd_linear_out. */
size_t fd_linear_noalloc_scratch_bytes(void);
/* Health of the scratch (no counterpart in the reference).  A call whose
 * bounded in-kernel wait expired (a stalled copy engine, a pre-empted GPU)
 * leaves invalid outputs, a non-zero status word and possibly half-counted
 * split-K counters in the shared scratch -- which would make every later call
 * on that device reduce the wrong blocks.  A caller without a workspace of
 * its own cannot reach that memory, so:
 *   fd_linear_noalloc_status: the status word after all work enqueued on
 *     `stream` so far (0: no wait expired); waits for `stream` to finish.
 *   fd_linear_noalloc_reset: zero the counters and the status word on
 *     `stream` (asynchronous, allocates nothing); the next call then starts
 *     from a clean scratch.
 * Both use the scratch of the current device. */
int fd_linear_noalloc_status(int32_t* status, void* stream);
int fd_linear_noalloc_reset(void* stream);
int fd_linear_out_noalloc(const void* x, int64_t sxm, int64_t sxk,
                          const void* w, int64_t swn, int64_t swk,
                          const void* bias, int32_t bias_dtype, int64_t sbias,
                          const void* row_add, int32_t ra_dtype, int64_t srm, int64_t srn,
                          void* y, int64_t sym, int64_t syn,
                          int32_t dtype, int32_t m, int64_t n, int64_t k, int32_t kind,
                          void* stream);

/* Workspace bytes fd_post_attn_mlp_out / fd_mlp_gate_up_out need (zero-filled
 * once, as above). */
size_t fd_post_attn_mlp_workspace_bytes(int32_t m, int64_t h, int64_t i);

/* Llama post-attention MLP for 1 <= m <= 16 contiguous rows of width h:
 *   normed  = round(rmsnorm(hidden) * norm_w)
 *   gate_up = round(normed @ w_gate_up^T)   (w_gate_up is [2i, h], gate above up)
 *   mid     = round(silu(gate) * up)
 *   out     = round(mid @ w_down^T + hidden)   (w_down is [h, i])
 * Two launches (RMSNorm + gate/up + SwiGLU, then down + residual; the second
 * programmatic-dependent on the first) instead of the reference's four.  add_residual = 0 drops "+ hidden";
 * out_dtype = FD_F32 stores the unrounded fp32 sum (a tensor-parallel rank's
 * partial before its allreduce), otherwise out_dtype must equal dtype.
 * w_gate_up / w_down may carry any row stride that is a multiple of 8
 * (k-stride 1); norm_w is f16, bf16 or f32.  The rounding points follow
 * post_attn_mlp_reference (reference reference.py:66-79).
 * Replaces post_attn_mlp's launches (reference ops.py:312-315). */
int fd_post_attn_mlp_out(const void* hidden, const void* norm_w, int32_t norm_dtype,
                         const void* w_gate_up, int64_t s_gu,
                         const void* w_down, int64_t s_down,
                         void* out, int32_t out_dtype, int32_t dtype,
                         int32_t m, int64_t h, int64_t i, float eps, int32_t kind,
                         int32_t add_residual, void* workspace, size_t workspace_bytes,
                         void* stream);

/* `layers` consecutive post_attn_mlp layers (layer l reads layer l-1's
 * output): norm_w, w_gate_up and w_down are HOST arrays of `layers` device
 * pointers with shared shapes, strides and dtypes.  Intermediate activations
 * live in the workspace and only the last layer's output is written to
 * `out`.  The workspace is fd_post_attn_mlp_workspace_bytes(m, h, i).
 * Two programmatic-dependent launches per layer.  With FD_STACK_PERSISTENT=1
 * in the environment and kind = FD_KIND_DOT, ONE persistent cooperative
 * kernel per 32 layers instead (one CTA per SM; the weight stream runs on
 * across layer and phase boundaries while grid-wide barriers order the
 * activations; status bit 16: a barrier wait expired) where the batch leaves
 * it at least 4 ring stages -- measured no faster on one B200, so not the
 * default.  Both give the same bits as one fd_post_attn_mlp_out call per layer.
 * Replaces a loop of post_attn_mlp calls (reference ops.py:283-315). */
/* Kernel launches one fd_post_attn_mlp_stack_out call of this shape makes
 * under the current environment (no counterpart in the reference). */
int fd_post_attn_mlp_stack_launches(int32_t layers, int32_t norm_dtype, int32_t m, int64_t h, int64_t i,
                                    int32_t kind);
int fd_post_attn_mlp_stack_out(const void* hidden, int32_t layers,
                               const void* const* norm_w, int32_t norm_dtype,
                               const void* const* w_gate_up, int64_t s_gu,
                               const void* const* w_down, int64_t s_down,
                               void* out, int32_t dtype, int32_t m, int64_t h, int64_t i,
                               float eps, int32_t kind, void* workspace,
                               size_t workspace_bytes, void* stream);

/* ---- tensor-parallel MLP over NVLink (no counterpart in the reference,
 * which has no multi-GPU code; this is its post_attn_mlp, ops.py:283-315,
 * split Megatron-style across `world` GPUs of one node).
 *
 * Every rank owns one exchange buffer of fd_tp_exchange_bytes(world, m_max, n)
 * bytes (n = hidden width, m_max = the largest batch it will carry, <= 16)
 * and maps every other rank's through CUDA IPC: fd_tp_exchange_alloc (zeroed
 * device memory), fd_tp_exchange_handle (64-byte IPC handle to share with the
 * other ranks), fd_tp_exchange_open / _close (map / unmap a peer's buffer),
 * fd_tp_exchange_free.  The buffers carry a round number, so a group must
 * call fd_post_attn_mlp_tp_out the same number of times on every rank, in
 * the same order. */
size_t fd_tp_exchange_bytes(int32_t world, int32_t m_max, int64_t n);
int fd_tp_exchange_alloc(int32_t world, int32_t m_max, int64_t n, void** buf);
int fd_tp_exchange_free(void* buf);
int fd_tp_exchange_handle(void* buf, void* handle);
int fd_tp_exchange_open(const void* handle, void** peer);
int fd_tp_exchange_close(void* peer);

/* One tensor-parallel post_attn_mlp layer on rank `rank` of `world`:
 * w_gate_up is this rank's [2*i, h] restack (its gate rows over the matching
 * up rows), w_down its [h, i] column slice; hidden [m, h] is replicated.
 * Launches the gate/up kernel, the down-projection kernel -- whose block
 * partials go straight into every rank's exchange buffer (`exchange` holds
 * world device pointers: this rank's buffer at [rank], the mapped peer
 * buffers elsewhere) -- and a kernel that waits (bounded) for all ranks'
 * partials, sums them in rank order and writes out = round(sum + hidden),
 * the same bits on every rank.  With FD_TP_FOLD=1 in the environment and
 * kind = FD_KIND_DOT, the CTA that finishes a block of the down projection
 * does that sum for its block instead: two launches, the same bits.  A wait that expires sets bit 8 of the
 * workspace status word.  Workspace: fd_post_attn_mlp_workspace_bytes(m, h, i). */
int fd_post_attn_mlp_tp_out(const void* hidden, const void* norm_w, int32_t norm_dtype,
                            const void* w_gate_up, int64_t s_gu,
                            const void* w_down, int64_t s_down,
                            void* out, int32_t dtype, int32_t m, int64_t h, int64_t i,
                            float eps, int32_t kind, int32_t rank, int32_t world,
                            void* const* exchange, int32_t m_max,
                            void* workspace, size_t workspace_bytes, void* stream);

/* `layers` consecutive tensor-parallel post_attn_mlp layers on rank `rank`
 * of `world` (no counterpart in the reference): the stack form of
 * fd_post_attn_mlp_tp_out, with norm_w, w_gate_up (this rank's [2*i, h]
 * restacks) and w_down (its [h, i] column slices) as HOST arrays of device
 * pointers; only the last layer's output is written to `out`, every rank
 * getting the same bits.  Three launches per layer (two with FD_TP_FOLD=1); with FD_STACK_PERSISTENT=1
 * in the environment and kind = FD_KIND_DOT (where the batch leaves at
 * least 4 ring stages), one persistent cooperative kernel per 32 layers -- per layer a gate/up phase, a down
 * phase whose block partials go to every rank's exchange buffer, and a
 * phase that sums the ranks' partials (bounded waits, status bit 8) and adds
 * the residual -- with no launch between layers (measured slower than the
 * per-layer launches on 2 B200s, so not the default).  The same exchange and
 * round-counting rules as
 * fd_post_attn_mlp_tp_out.  Workspace: fd_post_attn_mlp_workspace_bytes(m, h, i). */
/* Kernel launches of one fd_post_attn_mlp_out (tensor_parallel = 0) or
 * fd_post_attn_mlp_tp_out (1) call of this shape (no counterpart in the
 * reference): two, plus a norm kernel where the gate/up stage streams the
 * normalised rows (batches whose normalised rows would leave its shared-memory
 * ring shallow), plus the rank-sum kernel for tensor parallel. */
int fd_post_attn_mlp_layer_launches(int32_t m, int64_t h, int64_t i, int32_t norm_dtype, int32_t kind,
                                    int32_t tensor_parallel);
/* Kernel launches one fd_post_attn_mlp_tp_stack_out call of this shape makes
 * (i: this rank's share of the intermediate width). */
int fd_post_attn_mlp_tp_stack_launches(int32_t layers, int32_t norm_dtype, int32_t m, int64_t h, int64_t i,
                                       int32_t kind);
int fd_post_attn_mlp_tp_stack_out(const void* hidden, int32_t layers, const void* const* norm_w,
                                  int32_t norm_dtype, const void* const* w_gate_up, int64_t s_gu,
                                  const void* const* w_down, int64_t s_down, void* out, int32_t dtype,
                                  int32_t m, int64_t h, int64_t i, float eps, int32_t kind, int32_t rank,
                                  int32_t world, void* const* exchange, int32_t m_max, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* First kernel of fd_post_attn_mlp_out on its own: mid[m, i] (contiguous) =
 * round(silu(gate) * up) of the RMSNorm'd hidden rows.  Replaces the
 * rms_norm -> linear_decode -> swiglu launches of post_attn_mlp (reference
 * ops.py:312-315). */
int fd_mlp_gate_up_out(const void* hidden, const void* norm_w, int32_t norm_dtype,
                       const void* w_gate_up, int64_t s_gu, void* mid, int32_t dtype,
                       int32_t m, int64_t h, int64_t i, float eps, int32_t kind,
                       void* workspace, size_t workspace_bytes, void* stream);

/* out[j] = round(partial[j] + residual[j]) for n contiguous elements: the
 * residual add after a tensor-parallel allreduce of fp32 partials (the
 * "+ hidden" of reference ops.py:315, moved after the reduction). */
int fd_residual_add_out(const float* partial, const void* residual, void* out,
                        int32_t dtype, int64_t n, void* stream);

/* dst[:bytes] = src[:bytes], 16-byte vectorised when both are 16-byte aligned.
 * The in-process copy roof; replaces launch_copy (reference kernels.py:849-852). */
int fd_copy(void* dst, const void* src, size_t bytes, void* stream);

/* c = a + b * scale over n elements of dtype (f16/bf16/f32), fp32 math.
 * Replaces launch_triad (reference kernels.py:855-858). */
int fd_triad(const void* a, const void* b, void* c, int64_t n, int32_t dtype,
             float scale, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FD_B200_H */
