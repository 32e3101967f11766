/*
 * umic_b200.h -- C ABI of the B200 (sm_100a) fused-inference hot path.
 *
 * Every entry point:
 *   - takes raw device pointers, element strides (in elements, not bytes) and a
 *     cudaStream_t (passed as void*; NULL = legacy default stream);
 *   - launches asynchronously on that stream, performs no host synchronisation
 *     and no device allocation, so it is safe inside CUDA-graph capture;
 *   - returns 0 on success or one of the UMIC_ERR_* codes below. The code is
 *     decided on the host before launch (shape / stride / alignment checks) or
 *     comes from the launch itself. umic_last_error_message() gives a one-line
 *     reason for the last non-zero return on the calling thread.
 *
 * Tensors are bf16 unless a dtype argument says otherwise. "Rows" are the
 * flattened leading dimensions; the last dimension must be contiguous.
 *
 * Each function names the reference interface it replaces
 * (soonhong99/umic-alpamayo, paths relative to that project's root).
 */
#ifndef UMIC_B200_H_
#define UMIC_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define UMIC_API __attribute__((visibility("default")))
#else
#define UMIC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define UMIC_OK 0
#define UMIC_ERR_INVALID_ARG 1  /* null pointer, negative or zero size */
#define UMIC_ERR_UNSUPPORTED 2  /* shape the kernel does not handle */
#define UMIC_ERR_ALIGNMENT 3    /* pointer or stride breaks a 16-byte rule */
#define UMIC_ERR_LAUNCH 4       /* CUDA reported an error at launch */
#define UMIC_ERR_OVERFLOW 5     /* KV append past the buffer capacity */
#define UMIC_ERR_DEVICE 6       /* no sm_100 device / driver entry point */

/* Device-side error bits, read with umic_device_errors(). */
#define UMIC_DEVERR_KV_OVERFLOW 1u   /* device-position KV append out of range */
#define UMIC_DEVERR_WAIT_TIMEOUT 2u  /* a bounded mbarrier wait ran out */

/* dtype codes for optional fp32 side inputs */
#define UMIC_DTYPE_BF16 0
#define UMIC_DTYPE_FP32 1

/* GEMV flags */
#define UMIC_GEMV_WEIGHTS_READY 1u /* weights not written by the preceding stream op */

/* GEMM epilogues */
#define UMIC_EPI_NONE 0
#define UMIC_EPI_GELU_ERF 1   /* 0.5*x*(1+erf(x/sqrt2)), linear.py:83-86 */
#define UMIC_EPI_GELU_TANH 2  /* tanh approximation (HF gelu_pytorch_tanh) */

/* ---- library ------------------------------------------------------------ */

/* ABI version: bumps when a signature changes. */
UMIC_API int umic_abi_version(void);

/* One-line reason for the last non-zero return on this thread ("" if none). */
UMIC_API const char* umic_last_error_message(void);

/* Makes `device` the current device of this library's CUDA runtime for the
 * calling thread (the library links its own runtime; the host wrapper calls
 * this when a tensor lives on another GPU than the previous call's).
 * No reference counterpart: the reference runs on one device. */
UMIC_API int umic_set_device(int device);

/* Reads the device-side error word of the current device into *flags
 * (synchronises the device). If clear != 0 the word is reset to 0.
 * No reference counterpart: the reference raises Python exceptions only. */
UMIC_API int umic_device_errors(uint32_t* flags, int clear);

/* Test hook of the bounded-wait abort path. Arms the NEXT launch of one kernel
 * family in this process (kernel = 1: the tensor-core GEMM, umic_gemm / umic_gemm_ws /
 * umic_gemm_gate_silu_mul; 2: the streaming GEMV engine): in that launch CTA 0 announces
 * the bytes of its first shared-memory stage but never loads them, and every bounded wait
 * of the launch gives up after wait_limit_cycles SM cycles instead of about 5 s. The
 * stalled CTA (and its pair partner) then sets UMIC_DEVERR_WAIT_TIMEOUT, lets its copies
 * in flight land, frees its tensor memory and exits; that launch's output is undefined,
 * and the counters in the workspace of that launch (streaming GEMV, split-K GEMM) may be
 * left non-zero (zero the workspace before its next use). Calls made after it run
 * normally. The arm is consumed by the first matching launch. kernel = 3 is not a
 * stall: the next streaming-GEMV launch merges every row block split between two CTAs
 * through the general path (count, then sum), never the shortcut that takes an already
 * posted partner partial, so tests can compare the two merges bit for bit
 * (wait_limit_cycles must be positive and is otherwise ignored).
 * No reference counterpart: the reference has no device-side waits. */
UMIC_API int umic_debug_stall(int kernel, int64_t wait_limit_cycles);

/* ---- RMSNorm family (src/umic/kernels/rmsnorm.py) ------------------------ */

/* y = bf16(x * rsqrt(mean(x^2) + eps) * w), fp32 inside.
 * Replaces rmsnorm_triton / _rmsnorm_kernel (rmsnorm.py:32-73).
 * w_dtype: UMIC_DTYPE_BF16 or UMIC_DTYPE_FP32. */
UMIC_API int umic_rmsnorm(const void* x, int64_t x_row_stride, const void* w, int w_dtype,
                 void* y, int64_t y_row_stride, int64_t rows, int64_t n, float eps,
                 void* stream);

/* s = x + r (fp32); summed = bf16(s); normed = bf16(s * rsqrt(mean(s^2)+eps) * w).
 * Replaces add_rmsnorm_triton / _add_rmsnorm_kernel (rmsnorm.py:75-134). */
UMIC_API int umic_add_rmsnorm(const void* x, int64_t x_row_stride, const void* r,
                     int64_t r_row_stride, const void* w, int w_dtype, void* normed,
                     int64_t normed_row_stride, void* summed, int64_t summed_row_stride,
                     int64_t rows, int64_t n, float eps, void* stream);

/* y = bf16(base + alpha * (x * rsqrt(mean(x^2) + eps) * w)), fp32 inside, one
 * rounding: RMSNorm with an axpy epilogue. The flow sampler's Euler update
 * x <- x + dt * v, where the velocity v is the action expert's final RMSNorm output,
 * runs as this one pass (v is never stored). y may be base itself (same pointer and
 * row stride); row strides must be positive.
 * Replaces the expert's final norm (_patched_rmsnorm_forward, integrate.py:134-141)
 * together with P9 ode_step, x <- x + dt*v (docs/260610_01_umic_design_ko.md:72),
 * which the reference lists but never builds. */
UMIC_API int umic_rmsnorm_axpy(const void* x, int64_t x_row_stride, const void* w, int w_dtype,
                               const void* base, int64_t base_row_stride, float alpha, void* y,
                               int64_t y_row_stride, int64_t rows, int64_t n, float eps,
                               void* stream);

/* ---- LayerNorm family (src/umic/kernels/layernorm.py) -------------------- */

/* y = bf16((x - mean) * rsqrt(var + eps) * w + b), fp32 inside; w and b share
 * w_dtype. Replaces layernorm_triton / _layernorm_kernel (layernorm.py:31-68). */
UMIC_API int umic_layernorm(const void* x, int64_t x_row_stride, const void* w, const void* b,
                   int w_dtype, void* y, int64_t y_row_stride, int64_t rows, int64_t n,
                   float eps, void* stream);

/* add + LayerNorm with two outputs (normed, summed).
 * Replaces add_layernorm_triton / _add_layernorm_kernel (layernorm.py:70-124). */
UMIC_API int umic_add_layernorm(const void* x, int64_t x_row_stride, const void* r,
                       int64_t r_row_stride, const void* w, const void* b, int w_dtype,
                       void* normed, int64_t normed_row_stride, void* summed,
                       int64_t summed_row_stride, int64_t rows, int64_t n, float eps,
                       void* stream);

/* ---- rotary embedding, in place (src/umic/kernels/rope.py) --------------- */

/* In-place rotate-half RoPE on q and (optionally) k:
 *   out[d]       = x[d]*cos[d]         - x[d+D/2]*sin[d]
 *   out[d+D/2]   = x[d+D/2]*cos[d+D/2] + x[d]*sin[d+D/2]      (d < D/2)
 * fp32 inside, one bf16 rounding. q is indexed [batch, seq, head, dim] through
 * (q_sb, q_ss, q_sh) element strides with dim contiguous; k likewise (k may be
 * NULL with hk = 0). cos/sin are [batch, seq, dim] through (c_sb, c_ss), in
 * cos_dtype (bf16 for HF text RoPE, fp32 for HF vision RoPE); c_sb may be 0 to
 * broadcast one table over the batch.
 * Replaces _rope_kernel/_apply_one (rope.py:31-76), apply_rotary_vision_triton
 * (rope.py:78-84) and the text path of make_text_rope (rope.py:86-107), which
 * were out-of-place. */
UMIC_API int umic_rope_inplace(void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh, int32_t hq,
                      void* k, int64_t k_sb, int64_t k_ss, int64_t k_sh, int32_t hk,
                      const void* cos, const void* sin, int64_t c_sb, int64_t c_ss,
                      int cos_dtype, int64_t batch, int64_t seq, int32_t head_dim,
                      void* stream);

/* ---- KV cache (src/umic/cache.py) ----------------------------------------- */

/* Writes n_new tokens of k_new / v_new into the preallocated buffers at token
 * position pos (host value) or *dpos (device int64, read at execution time so a
 * captured graph can replay at a moving position; pass dpos = NULL to use pos).
 * Buffers are [batch, heads, capacity, head_dim] through (buf_sb, buf_sh,
 * buf_ss) element strides; k_new / v_new are [batch, heads, n_new, head_dim]
 * through their own strides. A host position past capacity returns
 * UMIC_ERR_OVERFLOW without launching; a device position past capacity skips
 * the write and sets UMIC_DEVERR_KV_OVERFLOW.
 * Replaces InplaceLayer.update's writes (cache.py:50-80: slice assignment and the
 * graph-mode index_copy_ at cache.py:59-60). */
UMIC_API int umic_kv_append(void* k_buf, void* v_buf, int64_t buf_sb, int64_t buf_sh,
                   int64_t buf_ss, int64_t capacity, const void* k_new, int64_t kn_sb,
                   int64_t kn_sh, int64_t kn_ss, const void* v_new, int64_t vn_sb,
                   int64_t vn_sh, int64_t vn_ss, int64_t batch, int32_t heads,
                   int64_t n_new, int32_t head_dim, int64_t pos, const int64_t* dpos,
                   void* stream);

/* Attention input in one pass: per-head RMSNorm (weights q_weight / k_weight
 * [head_dim], eps q_eps / k_eps; NULL weight = no norm) and rotate-half RoPE of q
 * and k, then the K/V write. q and k are [batch, seq, heads, head_dim] through
 * their (sb, ss, sh) element strides; v likewise with hk heads. q is rotated in
 * place. With k_buf != NULL the normalised, rotated k and the unchanged v are
 * written to the cache buffers [batch, hk, capacity, head_dim] (strides buf_*)
 * at token position pos (host) or *dpos (device), with the same overflow rules
 * as umic_kv_append; with k_buf == NULL k is written back in place and v is not
 * touched. cos/sin as in umic_rope_inplace. head_dim 64, 128 or 256.
 * Replaces, as one kernel, q_norm / k_norm (_patched_rmsnorm_forward,
 * integrate.py:134-141), apply_rotary_pos_emb (rope.py:86-107) and the cache
 * write of InplaceLayer.update (cache.py:59-60, 69-70). */
UMIC_API int umic_qk_norm_rope_kv(
    void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh, int32_t hq, void* k, int64_t k_sb,
    int64_t k_ss, int64_t k_sh, const void* v, int64_t v_sb, int64_t v_ss, int64_t v_sh,
    int32_t hk, const void* q_weight, const void* k_weight, int w_dtype, float q_eps,
    float k_eps, const void* cos, const void* sin, int64_t c_sb, int64_t c_ss, int cos_dtype,
    void* k_buf, void* v_buf, int64_t buf_sb, int64_t buf_sh, int64_t buf_ss, int64_t capacity,
    int64_t pos, const int64_t* dpos, int64_t batch, int64_t seq, int32_t head_dim,
    void* stream);

/* ---- attention over a cached prefix -------------------------------------- */

/* out = softmax(scale * q . k^T, masked) . v with grouped-query heads, for few
 * query rows per KV head over a long key prefix (the flow expert's action tokens
 * over its cached prefix), or for one query head per KV head over 128-token tiles
 * (the ViT's per-image attention). q [batch, hq, t, d] through strides (q_sb, q_sh,
 * q_st); k, v [batch, hkv, lk, d] through (sb, sh, sl) -- e.g. the prefix view of
 * an in-place cache buffer; out [batch, hq, t, d] through (o_sb, o_sh, o_st).
 * mask_bits: the mask as packed by umic_mask_pack_bits -- key k of (b, head, token)
 * attends iff bit k % 32 of word b*m_sb + head*m_sh + token*m_st + k / 32 is set (word
 * strides; 0 broadcasts) -- or NULL for no mask; rows that attend to nothing come
 * out as zeros. Covers head_dim 64..128 (a multiple of 8), hq a multiple of hkv, and
 * either (hq / hkv) * t <= 128 with t a multiple of 8 (one CTA per batch and kv head)
 * or hq == hkv with any t (one CTA per 128 tokens, e.g. the ViT's 1024 patches per
 * image), 16-byte aligned bases and strides that are multiples of 8 elements; other
 * shapes return UMIC_ERR_UNSUPPORTED / UMIC_ERR_ALIGNMENT and the caller keeps its
 * own attention. No kernel counterpart in the reference: it leaves
 * this attention to torch SDPA inside the HF attention forward that its flow-cache
 * hook serves (src/umic/integrate.py:715-756); this replaces that SDPA call. */
UMIC_API int umic_attention_rows(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st,
                                 const void* k, int64_t k_sb, int64_t k_sh, int64_t k_sl,
                                 const void* v, int64_t v_sb, int64_t v_sh, int64_t v_sl,
                                 const uint32_t* mask_bits, int64_t m_sb, int64_t m_sh,
                                 int64_t m_st, void* out, int64_t o_sb, int64_t o_sh,
                                 int64_t o_st, int64_t batch, int64_t hq, int64_t hkv, int64_t t,
                                 int64_t lk, int64_t head_dim, float scale, void* stream);

/* Packs a boolean attention mask (bytes, nonzero = attend; element (b, h, token, key)
 * at b*sb + h*sh + token*st + key) into bits for umic_attention_rows: word w of row
 * (b, h, token), at bits + b*wb + h*wh + token*wt (word strides), holds keys
 * 32 w .. 32 w + 31, key 32 w + i in bit i; bits past lk are zero. Each row needs
 * ceil(lk / 32) words. Part of umic_attention_rows's path, no reference counterpart
 * (the reference hands the byte mask to torch SDPA). */
UMIC_API int umic_mask_pack_bits(const void* mask, int64_t sb, int64_t sh, int64_t st,
                                 int64_t batch, int64_t heads, int64_t t, int64_t lk,
                                 uint32_t* bits, int64_t wb, int64_t wh, int64_t wt,
                                 void* stream);

/* ---- projections (src/umic/kernels/linear.py, fused_ffn.py) -------------- */

/* Row-count regime below FUSE_MIN_ROWS (integrate.py:27-30): HBM-bound GEMV,
 * y[m, n] = sum_k x[m, k] * w[n, k] (+ bias[n]); m < 64. w is [n, k] row-major
 * (nn.Linear layout). Replaces the cuBLAS fallback of _patched_linear_forward
 * (integrate.py:104-105). bias may be NULL.
 *
 * workspace: scratch of at least umic_gemv_workspace_bytes(n) bytes, 256-byte
 * aligned, zero-filled before its first use; every call leaves it zeroed again.
 * With a workspace, m <= 16 runs the streaming engine (TMA-fed, one CTA per SM,
 * deterministic fixed-order reduction, programmatic dependent launch); with
 * workspace == NULL (or m > 16) the cluster split-K engine runs, which needs no
 * scratch. Calls sharing one workspace must be ordered on one stream: overlapping
 * calls race on it. The same applies to the two calls below.
 *
 * flags: 0 or UMIC_GEMV_WEIGHTS_READY. The streaming engine is launched with
 * programmatic stream serialization, so it may start while the previous kernel in
 * the stream is finishing; x, y, bias and the workspace are only touched after that
 * kernel completes. With UMIC_GEMV_WEIGHTS_READY the caller promises that the
 * weights are not written by the operation enqueued just before this call, and the
 * weight stream begins at once (e.g. model parameters inside a forward pass). */
UMIC_API int umic_gemv(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* bias,
                       void* y, int64_t ldy, int64_t m, int64_t n, int64_t k, void* workspace,
                       size_t workspace_bytes, uint32_t flags, void* stream);

/* umic_gemv without a caller workspace and without any allocation. No counterpart
 * in the reference (its GEMVs go through torch, which allocates freely); this is an
 * extra entry for hosts that cannot allocate device memory when they call in: an
 * embedded driving stack that reserves all device memory at start-up and forbids
 * cudaMalloc inside its real-time control loop (cudaMalloc and cudaFree may
 * synchronise the device and have unbounded latency), or an FFI binding whose
 * runtime owns device memory in its own pool and has no way to hand a workspace
 * through. The streaming engine runs on a scratch array that is part of the
 * library image: a 256-byte-aligned __device__ array of 4 MB + 64 KB that every
 * GPU which loads the library holds until the process exits. Its device address
 * is looked up with cudaGetSymbolAddress by the first call on each device (with
 * that device current); make that first call before any stream capture.
 * Limits: 1 <= m <= 16, n <= 1048576 weight rows, at most 256 SMs; larger calls
 * return UMIC_ERR_UNSUPPORTED with the limit in the message. The array keeps the
 * last call's contents, so each call first clears its row-block counters with a
 * stream-ordered cudaMemsetAsync and then launches in plain stream order. All
 * calls on one device share the array: calls that overlap on the GPU (other
 * streams or threads) race on it and must be serialised by the caller. Same
 * result as umic_gemv with a workspace, bit for bit. */
UMIC_API int umic_gemv_noalloc(const void* x, int64_t ldx, const void* w, int64_t ldw,
                               const void* bias, void* y, int64_t ldy, int64_t m, int64_t n,
                               int64_t k, void* stream);

/* umic_gemv with the residual add in its epilogue: y = x . w^T (+ bias) + res, with
 * res [m, n] bf16 (leading dimension ldres, 16-byte aligned); y may be res itself
 * (same pointer and leading dimension: each element is read before it is written). The
 * streaming engine only (1 <= m <= 16, a workspace as for umic_gemv); other shapes
 * return UMIC_ERR_UNSUPPORTED and the caller keeps its unfused path. Replaces, in a
 * decode step, down_proj followed by the residual add (integrate.py:180-209, the
 * decoder-layer forward whose tail this is, and the Linear it calls). */
UMIC_API int umic_gemv_residual(const void* x, int64_t ldx, const void* w, int64_t ldw,
                                const void* bias, const void* res, int64_t ldres, void* y,
                                int64_t ldy, int64_t m, int64_t n, int64_t k, void* workspace,
                                size_t workspace_bytes, uint32_t flags, void* stream);

/* Bytes of workspace the streaming engine needs for `rows` weight rows in one call
 * (for umic_gemv_multi: the sum of n_i) on the current device. */
UMIC_API size_t umic_gemv_workspace_bytes(int64_t rows);

/* Up to 3 GEMVs sharing x in one launch (e.g. the q, k and v projections of a
 * decode step): y_i = x . w_i^T (+ bias_i) for i < count, with w_i [n_i, k],
 * y_i [m, n_i] (leading dimension ldy_i). Every n_i but the last must be a
 * multiple of 16 (of 64 for the streaming engine; otherwise the cluster engine
 * runs). Host arrays of length count; bias may be NULL (or hold NULLs).
 * No reference counterpart as one call: replaces the q_proj / k_proj / v_proj
 * calls of one decode step (integrate.py:98-107 and the cuBLAS k/v sites). */
UMIC_API int umic_gemv_multi(const void* x, int64_t ldx, int32_t count, const void* const* w,
                             const int64_t* ldw, const int64_t* n, const void* const* bias,
                             void* const* y, const int64_t* ldy, int64_t m, int64_t k,
                             void* workspace, size_t workspace_bytes, uint32_t flags,
                             void* stream);

/* h[m, n] = silu(x . wg[n]) * (x . wu[n]) for m < 64 rows.
 * Replaces the small-row branch of _fused_mlp_forward (integrate.py:48-50). */
UMIC_API int umic_gemv_gate_silu_mul(const void* x, int64_t ldx, const void* wg, const void* wu,
                                     int64_t ldw, void* h, int64_t ldh, int64_t m, int64_t n,
                                     int64_t k, void* workspace, size_t workspace_bytes,
                                     uint32_t flags, void* stream);

/* Tensor-core (tcgen05 + TMEM, TMA-fed) GEMM: y = epi(x . w^T + bias) + residual.
 * x [m, k], w [n, k] (both K-major), y [m, n]. bias / residual may be NULL.
 * epilogue: UMIC_EPI_*. Requires k % 8 == 0, n % 8 == 0, leading dimensions that
 * are multiples of 8 elements and 16-byte aligned base pointers.
 * Replaces linear_triton / _linear_kernel (linear.py:32-145). */
UMIC_API int umic_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* bias,
              const void* residual, int64_t ldr, void* y, int64_t ldy, int64_t m,
              int64_t n, int64_t k, int epilogue, void* stream);

/* umic_gemm with a caller workspace that enables split-K for shapes whose output tiles
 * would leave most of the GPU idle (at most half the CTA pairs busy: e.g. the flow
 * expert's q/o/down projections over 4 episodes, 256 rows x 2048 columns = 8 tiles for
 * 74 CTA pairs). Each tile's k-blocks are then cut into up to 8 ranges of at least 4
 * k-blocks, one work unit per CTA pair (per CTA for m <= 128). A unit owns whole 32-column
 * chunks of its tile: it writes its fp32 partials of the chunks the other units own to the
 * workspace, waits until they have written theirs, sums its own chunks over all partials
 * in range order (deterministic) and runs the epilogue (bias, GELU, residual) on them.
 * The units wait for one another, so a launch assumes all of them resident at once (there
 * are never more units than CTA pairs or CTAs); a kernel on another stream that holds SMs
 * meanwhile can keep a unit out past the wait limit, and the call then ends with
 * UMIC_DEVERR_WAIT_TIMEOUT set instead of hanging. Other shapes run exactly as
 * umic_gemm. workspace: at least
 * umic_gemm_workspace_bytes(m, n, k) bytes (0 when no split applies), 256-byte aligned,
 * zero-filled before its first use; every call leaves its counters at zero, except a call
 * that set UMIC_DEVERR_WAIT_TIMEOUT: zero the workspace again after one. Calls sharing
 * a workspace must be ordered on one stream. Replaces linear_triton (linear.py:118-145)
 * for the small-row shapes the reference sent to cuBLAS. */
UMIC_API int umic_gemm_ws(const void* x, int64_t ldx, const void* w, int64_t ldw,
                          const void* bias, const void* residual, int64_t ldr, void* y,
                          int64_t ldy, int64_t m, int64_t n, int64_t k, int epilogue,
                          void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of workspace umic_gemm_ws needs for this shape on the current device (0: the
 * shape fills the GPU without splitting). */
UMIC_API size_t umic_gemm_workspace_bytes(int64_t m, int64_t n, int64_t k);

/* Dual-accumulator tensor-core GEMM with the SwiGLU epilogue in registers:
 * h = silu(x . wg^T) * (x . wu^T); the gate and up products never reach HBM.
 * wg / wu are [n, k] (nn.Linear layout). Same alignment rules as umic_gemm.
 * Replaces gate_silu_mul_triton / _gate_silu_mul_kernel (fused_ffn.py:48-118). */
UMIC_API int umic_gemm_gate_silu_mul(const void* x, int64_t ldx, const void* wg, int64_t ldwg,
                            const void* wu, int64_t ldwu, void* h, int64_t ldh,
                            int64_t m, int64_t n, int64_t k, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* UMIC_B200_H_ */
