/*
 * hspmn_sm100.h - C ABI of libhspmn_sm100.so, the B200 (sm_100a) kernels of
 * the HSPMN v2.1 contextual-stream inference path:
 *
 *   (fp32 gate ->) router top-K  ->  gather selected queries  ->  SQDK causal attention
 *                 ->  scatter back into the [B,S,D] stream
 *
 * and, for training, the backward of the SQDK attention.
 *
 * Conventions
 *   - All buffers are device memory allocated by the caller; the library never
 *     allocates and never synchronises the stream it is given.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default).
 *   - Functions return HSPMN_OK (0) or a negative HSPMN_ERR_* code; the
 *     launch is skipped when validation fails.
 *   - Faults the host cannot see without a sync (query positions out of
 *     range, unsorted indices given to the scatter, a pipeline wait that gave
 *     up) set bits in a per-device flag word read by hspmn_device_errors().
 *   - Strides are in ELEMENTS for typed tensors and in BYTES for the
 *     row-copy kernels (gather/scatter move opaque rows).
 *
 * Element types: HSPMN_F32, HSPMN_F16, HSPMN_BF16.
 */
#ifndef HSPMN_SM100_H_
#define HSPMN_SM100_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define HSPMN_API __attribute__((visibility("default")))
#else
#define HSPMN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum hspmn_dtype { HSPMN_F32 = 0, HSPMN_F16 = 1, HSPMN_BF16 = 2 };

enum hspmn_status {
  HSPMN_OK = 0,
  HSPMN_ERR_INVALID = -1,     /* null pointer, bad size or shape */
  HSPMN_ERR_DTYPE = -2,       /* element type not supported by this entry point */
  HSPMN_ERR_ALIGN = -3,       /* pointer / stride alignment the kernel needs */
  HSPMN_ERR_UNSUPPORTED = -4, /* head_dim, head grouping or gate row length outside the kernel's range */
  HSPMN_ERR_CUDA = -5,        /* a CUDA runtime call or the launch failed */
  HSPMN_ERR_DEVICE = -6,      /* current device is not an sm_100 part */
  HSPMN_ERR_SCRATCH = -7      /* shape needs more scratch than hspmn_sqdk_fwd_noalloc holds */
};

/* bits of the device-side flag word */
#define HSPMN_DEVERR_POSITION 1u /* a query/selected position outside [0, S) */
#define HSPMN_DEVERR_UNSORTED 2u /* indices not ascending where an entry point requires it (scatter, backward) */
#define HSPMN_DEVERR_TIMEOUT 4u  /* a bounded pipeline wait in attention gave up */

/* Library version, major*10000 + minor*100 + patch. */
HSPMN_API int hspmn_version(void);

/* Static text for a status code. */
HSPMN_API const char* hspmn_strerror(int status);

/*
 * Router selection. Replaces the eval-mode part of TopKRouter.forward,
 * hspmn_v2_1.py:98,104-105,112-120:
 *   noisy[b,s] = round_to(noisy_dtype, logits[b,s] / temp)
 *   keep the K largest noisy values of each row (NaN largest; equal values:
 *   lower position first), write their positions ascending into
 *   indices[b, 0..K) and mask[b,s] = 1 if s was kept else 0.
 * logits: [B,S] of logits_dtype, row stride logits_rs (elements).
 * temp: one element of temp_dtype in device memory, or NULL for 1.
 * indices: int64 [B,K], row stride indices_rs. mask: uint8 [B,S], row
 * stride mask_rs; may be NULL.
 */
HSPMN_API int hspmn_router_topk(const void* logits, int logits_dtype, int64_t logits_rs,
                      const void* temp, int temp_dtype, int noisy_dtype,
                      int64_t B, int64_t S, int64_t K,
                      int64_t* indices, int64_t indices_rs,
                      uint8_t* mask, int64_t mask_rs, void* stream);

/*
 * Router gate with fp32 logits. Replaces the gate GEMV of TopKRouter.forward,
 * hspmn_v2_1.py:84,96 (logits = self.gate(x).squeeze(-1)), keeping the sum in
 * fp32 instead of rounding it to the module dtype:
 *   logits[b,s] = sum_d x[b,s,d] * weight[d] + bias[0]
 * Summation order is fixed (per-lane slot accumulators over 16-byte vectors,
 * a slot tree, a warp xor butterfly, bias last), so each logit depends only
 * on its row and is reproducible; feed the result to hspmn_router_topk with
 * logits_dtype HSPMN_F32.
 * x: [B,S,D] of x_dtype, strides x_sb, x_ss (elements), last dim contiguous.
 * weight: D contiguous elements of x_dtype; bias: one element of x_dtype or
 * NULL for 0. logits: float32 [B,S], row stride logits_rs.
 * Requires D a multiple of 8 (16-bit types) or 4 (f32), x and weight 16-byte
 * aligned and x_sb, x_ss multiples of 16 bytes (HSPMN_ERR_UNSUPPORTED /
 * HSPMN_ERR_ALIGN otherwise).
 */
HSPMN_API int hspmn_gate_logits(const void* x, int x_dtype, int64_t x_sb, int64_t x_ss,
                      const void* weight, const void* bias,
                      int64_t B, int64_t S, int64_t D,
                      float* logits, int64_t logits_rs, void* stream);

/*
 * Gather of the selected query rows, hspmn_v2_1.py:185-186:
 *   dst[b,i,:] = src[b, idx[b,i], :]     (row_bytes bytes per row)
 * src strides (bytes): src_sb per sequence, src_ss per position.
 * dst strides (bytes): dst_sb, dst_sk. idx: int64, row stride idx_sb.
 */
HSPMN_API int hspmn_gather_rows(const void* src, int64_t src_sb, int64_t src_ss,
                      const int64_t* idx, int64_t idx_sb,
                      void* dst, int64_t dst_sb, int64_t dst_sk,
                      int64_t B, int64_t S, int64_t K, int64_t row_bytes,
                      void* stream);

/*
 * Scatter into a zeroed stream, hspmn_v2_1.py:195-196:
 *   dst[b,s,:] = src[b,i,:] if idx[b,i] == s for some i, else 0
 * in one pass over dst (no separate zero fill). idx rows must be strictly
 * ascending, as the router writes them; violations set HSPMN_DEVERR_UNSORTED.
 */
HSPMN_API int hspmn_scatter_rows(const void* src, int64_t src_sb, int64_t src_sk,
                       const int64_t* idx, int64_t idx_sb,
                       void* dst, int64_t dst_sb, int64_t dst_ss,
                       int64_t B, int64_t S, int64_t K, int64_t row_bytes,
                       void* stream);

/*
 * Rotary embedding of the selected query rows, fused with their gather
 * (apply_rotary_pos_emb at hspmn_v2_1.py:66-68 on q, then hspmn_v2_1.py:185-186):
 *   dst[b,i,h,:] = rope(src[b, r, h, :], idx[b,i]),  r = idx[b,i] if
 *   src_by_position else i,
 *   rope(x, p)[d] = T(T(x[d]*cos[p,d]) + T(rot(x)[d]*sin[p,d])),
 *   rot(x) = cat(-x[hd/2:], x[:hd/2])
 * with the same per-operation rounding as the reference's three tensor ops,
 * so the rows are bit-identical to gathering after a full-tensor RoPE.
 * src rows: H*hd elements (strides in elements). idx row stride idx_sb may be
 * 0 (all sequences use one position list). cos/sin: [S, hd] tables of the
 * same dtype, row stride tab_ss. hd must be a multiple of 16 (bf16/f16)
 * or 8 (f32); rows, strides and tables 16-byte aligned.
 */
HSPMN_API int hspmn_rope_gather_rows(const void* src, int64_t src_sb, int64_t src_ss,
                                     int src_by_position, const int64_t* idx, int64_t idx_sb,
                                     const void* cos_tab, const void* sin_tab, int64_t tab_ss,
                                     void* dst, int64_t dst_sb, int64_t dst_sk,
                                     int64_t B, int64_t S, int64_t K, int64_t H, int64_t hd,
                                     int dtype, void* stream);

/*
 * Rotary embedding of every row of a [B,S,H,hd] tensor, row s at position
 * pos0 + s: the K side of apply_rotary_pos_emb (hspmn_v2_1.py:66-68, applied
 * at hspmn_v2_1.py:226-227) in one pass with no index array,
 *   dst[b,s,h,:] = rope(src[b,s,h,:], pos0 + s)
 * with rope() and its rounding as for hspmn_rope_gather_rows, so the rows are
 * bit-identical to the reference's three tensor ops. Row strides in elements
 * (src_sb, src_ss, dst_sb, dst_ss); each row's H*hd elements contiguous.
 * cos/sin: tables of tab_rows rows (pos0 + S <= tab_rows), row stride tab_ss.
 * dst may be src itself (same strides). hd a multiple of 16 (bf16/f16) or 8
 * (f32); rows, strides and tables 16-byte aligned.
 */
HSPMN_API int hspmn_rope_rows(const void* src, int64_t src_sb, int64_t src_ss,
                              const void* cos_tab, const void* sin_tab, int64_t tab_ss, int64_t tab_rows,
                              int64_t pos0, void* dst, int64_t dst_sb, int64_t dst_ss,
                              int64_t B, int64_t S, int64_t H, int64_t hd, int dtype, void* stream);

/*
 * In-place residual add of the selected rows (hspmn_v2_1.py:238 where every
 * unselected row of o_proj(scatter(...)) is zero):
 *   dst[b, idx[b,i], :] = T(dst[b, idx[b,i], :] + src[b,i,:])
 * row_elems elements per row; strides in elements; rows 16-byte aligned.
 * idx rows must not repeat a position (the router's never do).
 */
HSPMN_API int hspmn_scatter_add_rows(const void* src, int64_t src_sb, int64_t src_sk,
                                     const int64_t* idx, int64_t idx_sb,
                                     void* dst, int64_t dst_sb, int64_t dst_ss,
                                     int64_t B, int64_t S, int64_t K, int64_t row_elems,
                                     int dtype, void* stream);

/*
 * Sparse-query dense-key causal attention, the kernel behind
 * sparse_query_dense_key_attention (kernels_v2_1.py:141-180, compute at
 * kernels_v2_1.py:11-139), with grouped K/V heads as the reference's Flex
 * path defines them (hspmn_v2_1.py:212):
 *   o[b,i,h,:] = sum_{n <= idx[b,i]} softmax_n(sm_scale * q[b,i,h,:].k[b,n,g,:]) v[b,n,g,:]
 *   with g = h / (H / Hkv).
 * q, o: [B,K,H,hd]; k, v: [B,S,Hkv,hd]; strides in elements, innermost 1,
 * the others multiples of 16 bytes, bases 16-byte aligned.
 * dtype: HSPMN_BF16 or HSPMN_F16 (all of q, k, v, o). hd: a multiple of 8
 * up to 128 (computed on a 64- or 128-wide tile).
 * H % Hkv == 0 and H / Hkv <= 128.
 * workspace: launches with fewer 128-row tiles than two per SM split each
 * tile's keys over several CTAs and merge the partial results from a
 * caller-provided workspace of hspmn_sqdk_workspace_size() bytes (16-byte
 * aligned; NULL/0 when that size is 0). Launches that overlap on the GPU need
 * separate workspaces.
 */
HSPMN_API int hspmn_sqdk_fwd(const void* q, const int64_t* q_strides,
                   const void* k, const int64_t* k_strides,
                   const void* v, const int64_t* v_strides,
                   const int64_t* idx, int64_t idx_sb, int64_t idx_sk,
                   void* o, const int64_t* o_strides,
                   int64_t B, int64_t K, int64_t S, int64_t H, int64_t Hkv,
                   int64_t hd, int dtype, float sm_scale,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes hspmn_sqdk_fwd needs for this shape on the current device
 * (0: no split, no workspace; -1: the device could not be queried). */
HSPMN_API int64_t hspmn_sqdk_workspace_size(int64_t B, int64_t K, int64_t S, int64_t H,
                                            int64_t Hkv, int64_t hd);

/*
 * hspmn_sqdk_fwd without a workspace argument; no counterpart in the
 * reference, which allocates through PyTorch on every call.
 *
 * For callers that cannot allocate device memory at the moment they call:
 * a host without a device allocator of its own behind the C ABI (a plain C,
 * Go or Java caller that owns only the tensors it passes), or a caller inside
 * a region where an allocation would synchronise the device or fail. The
 * split-KV partials go to a static buffer of
 * HSPMN_SQDK_NOALLOC_SCRATCH_BYTES (32 MiB) that is part of the library's
 * module on each device; the call itself allocates nothing. That buffer is
 * device memory the library holds on every device its kernels are loaded on,
 * from load until exit, whether or not this entry point is ever called.
 *
 * Arguments, results and error codes are those of hspmn_sqdk_fwd, plus
 * HSPMN_ERR_SCRATCH, returned without launching anything, for shapes whose
 * hspmn_sqdk_workspace_size() exceeds HSPMN_SQDK_NOALLOC_SCRATCH_BYTES
 * (on a 148-SM B200 only launches with hd > 64 and 253 to 295 tiles of 128
 * rows can be).
 * Shapes with a workspace size of 0 do not touch the buffer.
 *
 * - Validation runs in the same order as in hspmn_sqdk_fwd, with
 *   HSPMN_ERR_SCRATCH where that function would find the workspace missing.
 * - The first call on a device whose launch uses the buffer (with that device
 *   current) looks up the buffer's device address and caches it; make such a
 *   call before any stream capture begins. The cached address is not
 *   refreshed after a cudaDeviceReset.
 * - Nothing in the buffer has to start at zero: every call writes each
 *   partial before it reads it.
 * - There is one buffer per device: calls on the same device whose work can
 *   overlap on the GPU (different streams without ordering between them, or
 *   several host threads) race on it and give wrong results. Order them on
 *   one stream, or use hspmn_sqdk_fwd with separate workspaces.
 */
#define HSPMN_SQDK_NOALLOC_SCRATCH_BYTES ((size_t)32 << 20)

HSPMN_API int hspmn_sqdk_fwd_noalloc(const void* q, const int64_t* q_strides,
                   const void* k, const int64_t* k_strides,
                   const void* v, const int64_t* v_strides,
                   const int64_t* idx, int64_t idx_sb, int64_t idx_sk,
                   void* o, const int64_t* o_strides,
                   int64_t B, int64_t K, int64_t S, int64_t H, int64_t Hkv,
                   int64_t hd, int dtype, float sm_scale, void* stream);

/*
 * hspmn_sqdk_fwd that also writes each row's log-sum-exp of the scaled scores
 * (natural log) to lse[b*lse_sb + i*lse_sk + h] (float32; lse_sk >= H), the
 * statistic hspmn_sqdk_bwd needs. Other arguments, results and errors as
 * hspmn_sqdk_fwd.
 */
HSPMN_API int hspmn_sqdk_fwd_lse(const void* q, const int64_t* q_strides,
                   const void* k, const int64_t* k_strides,
                   const void* v, const int64_t* v_strides,
                   const int64_t* idx, int64_t idx_sb, int64_t idx_sk,
                   void* o, const int64_t* o_strides,
                   float* lse, int64_t lse_sb, int64_t lse_sk,
                   int64_t B, int64_t K, int64_t S, int64_t H, int64_t Hkv,
                   int64_t hd, int dtype, float sm_scale,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of device workspace hspmn_sqdk_bwd needs (0 when K == 0). */
HSPMN_API int64_t hspmn_sqdk_bwd_workspace_size(int64_t B, int64_t K, int64_t H, int64_t hd);

/*
 * Backward of the SQDK attention. Replaces the gradient the reference's
 * training path takes through FlexAttention (hspmn_v2_1.py:200-216: mask
 * (q_idx >= kv_idx) & mask[b, q_idx] with enable_gqa, which is this
 * attention over the selected rows):
 *   dq = dL/dq [B,K,H,hd], dk = dL/dk and dv = dL/dv [B,S,Hkv,hd]
 * for the output gradient d_o [B,K,H,hd], given the forward's inputs, its
 * output o and its lse (from hspmn_sqdk_fwd_lse, dense [B,K,H]: lse_sb = K*H,
 * lse_sk = H). All tensors of `dtype` (bf16 or f16) with the last dimension
 * contiguous; q, k, v, d_o, dk, dv 16-byte aligned with 16-byte strides.
 * dk and dv are written in full (zero where no selected query sees a key).
 * workspace: hspmn_sqdk_bwd_workspace_size() bytes (16-byte aligned; holds
 * rowsum(dO * O) and an fp32 dq accumulator). hd: multiple of 8, <= 128;
 * H / Hkv <= 64. With K == 0 the query-side pointers may be null.
 * Each idx row must be ascending, as the router writes it: a key block finds
 * its first query by binary search. (The forward takes any order.) A row
 * found out of order sets HSPMN_DEVERR_UNSORTED; its gradients are then
 * incomplete.
 */
HSPMN_API int hspmn_sqdk_bwd(const void* q, const int64_t* q_strides,
                   const void* k, const int64_t* k_strides,
                   const void* v, const int64_t* v_strides,
                   const int64_t* idx, int64_t idx_sb, int64_t idx_sk,
                   const void* o, const int64_t* o_strides,
                   const void* d_o, const int64_t* do_strides,
                   const float* lse, int64_t lse_sb, int64_t lse_sk,
                   void* dq, const int64_t* dq_strides,
                   void* dk, const int64_t* dk_strides,
                   void* dv, const int64_t* dv_strides,
                   int64_t B, int64_t K, int64_t S, int64_t H, int64_t Hkv,
                   int64_t hd, int dtype, float sm_scale,
                   void* workspace, size_t workspace_bytes, void* stream);

/*
 * Read (and optionally clear) the current device's HSPMN_DEVERR_* flag word.
 * Synchronises `stream` first.
 */
HSPMN_API int hspmn_device_errors(unsigned* bits, int clear, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HSPMN_SM100_H_ */
