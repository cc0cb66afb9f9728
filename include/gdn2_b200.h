/*
 * gdn2_b200.h -- C ABI of the B200 (sm_100a) Gated DeltaNet-2 operator.
 *
 * This is the drop-in boundary for the reference operator
 *   make_blr_trainable(cfg, scale)(q, k, v, w, b, g, h0) -> (o, h_final)
 * of atomic_gdn2 (atomic_gdn2/pipeline.py:17-66), whose forward is the three
 * Pallas kernels build_scores / wy_solve_leafbatched / recompute_and_scan_slim
 * (pipeline.py:20-26) and whose backward is backward_mega (pipeline.py:38-47,
 * bwd/mega.py:61-79).  gdn2_fwd replaces `core_fwd` (pipeline.py:33-36) for one
 * segment, gdn2_bwd replaces `core_bwd` (pipeline.py:38-47).
 *
 * Plain C: raw device pointers, sizes and a CUDA stream (passed as void*).
 * Every buffer is allocated by the caller; the library owns no device memory.
 *
 * Layout: q, k, v, w, b, g, o, d_o and the six input gradients are (B, H, L, D)
 * tensors with unit stride along D, row stride D along L, and element strides
 * stride_b / stride_h along B / H (so segment views of a longer sequence need no
 * copy).  h0, h_final, d_hfinal and dh0 are contiguous (B, H, D, D) fp32 with
 * index [b][h][d_k][d_v].  o and h_final are fp32 (the reference returns the f32
 * kernel output, fwd/cd_slim.py:45); the six gradients are written in in_dtype
 * after the reference's final sanitize at 1e4 (pipeline.py:11-14, 44-47).
 */
#ifndef GDN2_B200_H
#define GDN2_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum gdn2_status {
  GDN2_OK = 0,
  /* Shape / dtype / config rejected before any launch.  Mirrors the reference's
   * ValueError paths (config.py:52-65, pipeline.py:54-55). */
  GDN2_ERR_INVALID_ARGUMENT = 1,
  /* A CUDA runtime call (launch, attribute set) failed. */
  GDN2_ERR_CUDA = 2,
  /* A configuration the reference accepts but this build does not implement. */
  GDN2_ERR_UNSUPPORTED = 3
} gdn2_status;

/* Dot-product precision modes (precision.py:8-37 plus one extra):
 *   HIGHEST  fp32-class products: 3 x tf32 (hi*hi + hi*lo + lo*hi)
 *   BF16X3   3 x bf16, the reference's dot_bf16x3 (precision.py:14-17)
 *   DEFAULT  1 x bf16 (jnp.dot at Precision.DEFAULT)
 *   TF32     1 x tf32 (no counterpart in the reference) */
typedef enum gdn2_precision {
  GDN2_PREC_HIGHEST = 0,
  GDN2_PREC_BF16X3 = 1,
  GDN2_PREC_DEFAULT = 2,
  GDN2_PREC_TF32 = 3
} gdn2_precision;

typedef enum gdn2_dtype { GDN2_F32 = 0, GDN2_BF16 = 1 } gdn2_dtype;

/* Bits of the device status word the kernels OR into (read it after the stream
 * has been synchronised). */
#define GDN2_DEV_TIMEOUT 1u        /* a bounded on-chip wait ran out (results invalid) */
#define GDN2_DEV_SPAN 2u           /* reserved: no longer raised (wide gate spans are computed exactly) */
#define GDN2_DEV_POSITIVE_GATE 4u  /* g > 0 seen: outside domain I-1 (domain.py:1-6) */

/* Operator descriptor.  Fields mirror BLRConfig (config.py:28-50) where they
 * affect the arithmetic; TPU tiling fields are not part of the ABI. */
typedef struct gdn2_desc {
  int32_t B, H, L, D;        /* L % bt == 0 (pipeline.py:54-55); D == 128 */
  int64_t stride_b;          /* element stride between batches of the (B,H,L,D) tensors */
  int64_t stride_h;          /* element stride between heads */
  int32_t bt;                /* chunk length, 128 */
  float scale;               /* output scale (make_blr_trainable's `scale`) */
  float wy_eps;              /* WY damping: A = (I + (1 - wy_eps) Akk)^-1 (fwd/solve.py:21-28) */
  float clip;                /* sanitize bound of intermediates (precision.py:50-51) */
  int32_t dot_mode;          /* gdn2_precision for scores / recompute / scan / B5 */
  int32_t solve_dot_mode;    /* gdn2_precision for the WY solve products */
  int32_t b3_dot_mode;       /* gdn2_precision for backward stages B1-B3 */
  int32_t in_dtype;          /* gdn2_dtype of q..g and of the six gradients */
} gdn2_desc;

/* Bytes of the residual buffer gdn2_fwd fills and gdn2_bwd reads for one call: the forward
 * intermediates the backward needs (scores Aqk, WY inverse A, wp, the state entering every chunk,
 * v_new).  The reference keeps gc, Aqk, A, h_pre_all, v_new_all (pipeline.py:25-26): 126.0 MB at
 * B4 H6 L2048 D128 against 125.8 MB here. */
size_t gdn2_residual_bytes(const gdn2_desc* desc);

/* Bytes of scratch gdn2_fwd needs beyond the residual buffer, dead once the call's work has run on
 * the stream (u = A (w v), the forward scan's state-transition images and additive terms). */
size_t gdn2_fwd_workspace_bytes(const gdn2_desc* desc);

/* Bytes of scratch gdn2_bwd needs beyond the residual buffer. */
size_t gdn2_bwd_workspace_bytes(const gdn2_desc* desc);

/* Forward over all L/bt chunks of one segment.  Replaces core_fwd
 * (pipeline.py:33-36 -> _fwd :20-26): gate cumsum, scores, WY solve,
 * recompute and the inter-chunk state scan.
 *   h0        (B,H,D,D) fp32 initial state, or NULL for zeros (pipeline.py:57)
 *   o         (B,H,L,D) fp32 output
 *   h_final   (B,H,D,D) fp32 final state
 *   residual  gdn2_residual_bytes(desc) bytes, 256-byte aligned (kept for gdn2_bwd)
 *   workspace gdn2_fwd_workspace_bytes(desc) bytes, 256-byte aligned (free after the call's work)
 *   dev_status device uint32 the kernels OR status bits into (never cleared by the library)
 *   stream    cudaStream_t; the work is ordered on it (see gdn2_set_batch_groups) */
gdn2_status gdn2_fwd(const gdn2_desc* desc, const void* q, const void* k, const void* v, const void* w,
                     const void* b, const void* g, const float* h0, float* o, float* h_final, void* residual,
                     void* workspace, uint32_t* dev_status, void* stream);

/* Backward of one segment.  Replaces core_bwd (pipeline.py:38-47 ->
 * backward_mega, bwd/mega.py:61-79).
 *   residual  the buffer gdn2_fwd filled for the same inputs
 *   h_final   (B,H,D,D) fp32, the h_final gdn2_fwd wrote for the same inputs (the state after
 *             the last chunk; kept by the caller as the forward's output, not in the residual)
 *   d_o       (B,H,L,D) fp32 cotangent of o (the reference casts do to f32, pipeline.py:42)
 *   d_hfinal  (B,H,D,D) fp32 cotangent of h_final, or NULL for zeros
 *   dq..dg    (B,H,L,D) gradients in in_dtype
 *   dh0       (B,H,D,D) fp32 gradient of h0
 *   workspace gdn2_bwd_workspace_bytes(desc) bytes, 256-byte aligned */
gdn2_status gdn2_bwd(const gdn2_desc* desc, const void* q, const void* k, const void* v, const void* w,
                     const void* b, const void* g, const void* residual, const float* h_final, const float* d_o,
                     const float* d_hfinal, void* dq, void* dk, void* dv, void* dw, void* db, void* dg, float* dh0,
                     void* workspace, uint32_t* dev_status, void* stream);

/* Batch groups (no counterpart in the reference; an execution setting, not part of the
 * arithmetic).  gdn2_fwd / gdn2_bwd split a call's B*H heads into up to n contiguous groups whose
 * launch sequences run on side streams the library owns, forked from the caller's stream by an
 * event and joined back to it before the call returns (capturable into a CUDA graph; the streams
 * are created by the first multi-group call on a device, which must not be under capture -- a call
 * under capture before that runs as one group).  A call whose B*H*(L/128) chunk-heads fit in one
 * wave of the GPU's multiprocessors runs as one group whatever n is.  Results do not depend on the
 * grouping.  n is clamped to [1, 8]; the initial value is the environment's GDN2_STREAMS, else 6.
 * Returns the previous value.
 * Scheduling: the state-scan launches of a call that is not being captured carry the device's
 * greatest launch priority (they are the short sequential links of each group's chain), so their
 * CTAs are dispatched ahead of pending CTAs of lower-priority streams, the caller's other work on
 * the device included; launches under capture keep the default priority. */
int32_t gdn2_set_batch_groups(int32_t n);
int32_t gdn2_get_batch_groups(void);

/* Human-readable name of a status code (static string). */
const char* gdn2_status_string(gdn2_status status);

/* Library self-test hook (no counterpart in the reference): one 128 x N x 128
 * tensor-core GEMM through the same shared-memory operand path the operator
 * kernels use.  C[m][n] = sum_k A'[m][k] B[k][n] with A' = A, or A' = A^T when
 * a_mode == 3.  A, B, C are contiguous fp32 device arrays (A 128x128, B 128xN,
 * C 128xN).  a_mode: 0 K-major slices, 1 MN-major slices, 2 whole-K K-major tile,
 * 3 whole-K K-major tile read through the transposed (MN-major) view (bf16 modes
 * only; tf32 returns GDN2_ERR_UNSUPPORTED).
 * b_mn: 0 K-major, 1 MN-major.  N in {32, 64, 128, 256}. */
gdn2_status gdn2_selftest_gemm(const float* A, const float* B, float* C, int32_t N, int32_t precision,
                               int32_t a_mode, int32_t b_mn, uint32_t* dev_status, void* stream);

/*
 * Self-test of the chunk kernels' operand staging engine (no reference counterpart): C = A B for
 * 128 x 128 fp32 matrices through one tensor-core product of the given precision, with A staged
 * as a K-major own-row (a_kind 0), K-major coalesced (1) or MN-major coalesced (2) operand and B
 * likewise (b_kind).  At and Bt are the transposes of A and B (row-major, device memory).
 */
gdn2_status gdn2_selftest_engine(const float* A, const float* At, const float* B, const float* Bt, float* C,
                                 int32_t precision, int32_t a_kind, int32_t b_kind, uint32_t* dev_status,
                                 void* stream);

/*
 * Failure-detection self-test (no reference counterpart; the reference's device code has no
 * waits): one warp waits, with the bounded on-chip wait every kernel of the library uses, on a
 * barrier phase that nothing completes.  The wait gives up after limit_cycles SM cycles
 * (0 < limit_cycles <= the library's own bound of 8e9), ORs GDN2_DEV_TIMEOUT into *dev_status
 * and stores the cycles it waited in *dev_cycles (-1 if the phase had completed).  Shows that a
 * stuck wait ends as a status bit the host reads while the context stays usable.
 */
gdn2_status gdn2_selftest_wait_timeout(uint32_t* dev_status, int64_t limit_cycles, int64_t* dev_cycles,
                                       void* stream);

/* Allocation-free forward (no counterpart in the reference).  Same arguments and results as
 * gdn2_fwd minus the residual and workspace buffers: both live in a fixed 64 MiB device array
 * inside the library, so the call performs no device allocation.  It is meant for callers that cannot
 * allocate at the point where they run the operator, such as runtime plugin / custom-call hooks
 * whose device memory is owned and planned by the host framework's allocator, and which receive
 * only a stream plus their input and output pointers.
 *   Limit: gdn2_residual_bytes(desc) rounded up to 256 bytes plus gdn2_fwd_workspace_bytes(desc)
 *   must be <= 64 MiB (about 96 chunk-heads of 128 tokens in
 *   the default modes, e.g. B=1, H=6, L=2048); larger problems are rejected with
 *   GDN2_ERR_INVALID_ARGUMENT before any launch; a descriptor gdn2_fwd rejects gets the same
 *   status here (GDN2_ERR_UNSUPPORTED for a chunk length or head size this build lacks).
 *   The first call on each device looks up the array's device address (cudaGetSymbolAddress);
 *   make that first call before any stream capture.  The address is kept for the life of the
 *   process: do not use this entry point across a cudaDeviceReset of that device.
 *   All calls on a device share the one array: calls that overlap on the GPU (different streams
 *   without ordering) race on it.  No state carries from one call to the next.
 *   Forward only: there is no residual to hand to gdn2_bwd. */
gdn2_status gdn2_fwd_noalloc(const gdn2_desc* desc, const void* q, const void* k, const void* v, const void* w,
                             const void* b, const void* g, const float* h0, float* o, float* h_final,
                             uint32_t* dev_status, void* stream);

/*
 * Fused layer prologue of the GDN-2 layer (atomic_gdn2/layer.py:31-40; the reference computes
 * it as XLA-fused jnp code, so there is no single reference function this replaces).
 * y is the layer's input projection, (B, L, 6, H, D) fp32 contiguous: the q, k, v, w, b, g
 * projections side by side per token.  gdn2_prologue_fwd writes the operator inputs as six
 * contiguous (B, H, L, D) fp32 tensors:
 *   q, k = y_q, y_k L2-normalised over D (eps 1e-6) when l2norm != 0, else unchanged;
 *   v, w = y_v, y_w;   b = sigmoid(y_b);   g = -min(softplus(y_g), g_max).
 * gdn2_prologue_bwd takes y and the six (B, H, L, D) gradients and writes dy in y's layout
 * (the activations are recomputed from y).  D must be 128 (GDN2_ERR_UNSUPPORTED otherwise);
 * every pointer must be 16-byte aligned (GDN2_ERR_INVALID_ARGUMENT otherwise).
 */
gdn2_status gdn2_prologue_fwd(const float* y, int64_t B, int64_t L, int64_t H, int64_t D, float g_max,
                              int32_t l2norm, float* q, float* k, float* v, float* w, float* b, float* g,
                              void* stream);
gdn2_status gdn2_prologue_bwd(const float* y, int64_t B, int64_t L, int64_t H, int64_t D, float g_max,
                              int32_t l2norm, const float* dq, const float* dk, const float* dv, const float* dw,
                              const float* db, const float* dg, float* dy, void* stream);

/* Profiling hook (no counterpart in the reference).  While enabled, every kernel launch of
 * gdn2_fwd / gdn2_bwd is bracketed by CUDA events recorded on the caller's stream.
 * gdn2_profile_collect synchronises on those events, writes per-kernel summed milliseconds and
 * launch counts for kernel ids [0, n) (GDN2_K_*), clears the record and returns the number of
 * timed launches. */
#define GDN2_K_FWD_INTRA 0
#define GDN2_K_FWD_SCAN 1
#define GDN2_K_FWD_OUT 2
#define GDN2_K_BWD_PRE 3
#define GDN2_K_BWD_SCAN 4
#define GDN2_K_BWD_INTRA 5
#define GDN2_K_COUNT 6
void gdn2_profile_enable(int32_t enable);
int32_t gdn2_profile_collect(float* ms, int32_t* counts, int32_t n);

#ifdef __cplusplus
}
#endif

#endif /* GDN2_B200_H */
