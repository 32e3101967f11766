// Attention input preparation in one pass: per-head RMSNorm of q and k, rotate-half
// RoPE of both, and the K/V write into the in-place cache.
//
// The reference runs this as separate steps -- q_norm and k_norm (one RMSNorm
// launch each, src/umic/integrate.py:134-141 applied to the per-head norms),
// apply_rotary_pos_emb (src/umic/kernels/rope.py:86-107) and the cache write
// (src/umic/cache.py:59-60, 69-70) -- each reading and writing q/k through HBM.
// Here a group of D/16 threads owns one head row of one token; each thread holds
// 8 elements of the first half (d0 = 8 * lane) and their 8 rotate-half partners
// (d0 + D/2), two 16-byte loads. The sum of squares is reduced with log2(D/16)
// shuffles, the normalised values stay in registers and the RoPE partner is
// already in the same thread, so the rotation needs no data exchange. q is
// written back in place; k (normalised, rotated) and v (copied) go straight to
// [b, h, pos + s, :] of the cache buffers, or k is written back in place when no
// cache buffer is given. Math in fp32, one bf16 rounding per output.
#include "common.cuh"

namespace umic {
namespace {

struct PrepArgs {
  __nv_bfloat16* q;
  __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const void* qw;
  const void* kw;
  const void* cos;
  const void* sin;
  __nv_bfloat16* kb;
  __nv_bfloat16* vb;
  const int64_t* dpos;
  uint32_t* err;
  int64_t q_sb, q_ss, q_sh;
  int64_t k_sb, k_ss, k_sh;
  int64_t v_sb, v_ss, v_sh;
  int64_t c_sb, c_ss;
  int64_t b_sb, b_sh, b_ss;
  int64_t capacity;
  int64_t pos;
  int64_t seq;
  int hq, hk;
  int w_dtype;
  float q_eps, k_eps;
};

template <bool kFp32>
__device__ __forceinline__ void load_table8(const void* base, int64_t idx, float (&f)[8]) {
  if constexpr (kFp32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + idx);
    const float4 a = __ldg(p), b = __ldg(p + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    unpack8(ld_cached(static_cast<const __nv_bfloat16*>(base) + idx), f);
  }
}

constexpr int kPrepThreads = 128;

// block = 128 threads = 128 / TPH head rows of one token, TPH = D / 16; grid =
// (seq, batch, ceil(rows / rows per block)). Row index r: [0, hq) q heads,
// [hq, hq+hk) k heads, then [hq+hk, hq+2hk) v heads when the K/V go to a cache.
// One token per thread with a small register footprint keeps many blocks resident,
// which is what bounds this kernel (the work per byte is a few dozen instructions).
template <int TPH, bool kCosFp32>
__global__ void __launch_bounds__(kPrepThreads) qk_prep_kernel(PrepArgs a) {
  allow_dependent_launch();
  wait_prerequisite();
  constexpr int kRowsPerBlock = kPrepThreads / TPH;
  constexpr int kHalfD = TPH * 8;  // D / 2
  const int sub = threadIdx.x % TPH;
  const int r = blockIdx.z * kRowsPerBlock + threadIdx.x / TPH;
  const int64_t s = blockIdx.x, b = blockIdx.y;
  const int rows = a.hq + (a.kb ? 2 * a.hk : a.hk);  // v rows only with a cache write
  const bool active = r < rows;
  int64_t pos = 0;
  if (a.kb) {
    pos = a.dpos ? *a.dpos : a.pos;
    if (pos < 0 || pos + a.seq > a.capacity) {
      if (threadIdx.x == 0 && s == 0 && b == 0 && blockIdx.z == 0 && a.err)
        atomicOr(a.err, UMIC_DEVERR_KV_OVERFLOW);
      return;  // uniform for the whole grid
    }
  }
  const int d0 = sub * 8;
  const bool is_q = active && r < a.hq;
  const bool is_v = active && r >= a.hq + a.hk;
  const bool is_k = active && !is_q && !is_v;
  const __nv_bfloat16* src = nullptr;
  __nv_bfloat16* dst = nullptr;
  if (is_q) {
    dst = a.q + b * a.q_sb + s * a.q_ss + r * a.q_sh + d0;
    src = dst;
  } else if (is_k) {
    const int h = r - a.hq;
    dst = a.k + b * a.k_sb + s * a.k_ss + h * a.k_sh + d0;
    src = dst;
    if (a.kb) dst = a.kb + b * a.b_sb + h * a.b_sh + (pos + s) * a.b_ss + d0;
  } else if (is_v) {
    const int h = r - a.hq - a.hk;
    src = a.v + b * a.v_sb + s * a.v_ss + h * a.v_sh + d0;
    dst = a.vb + b * a.b_sb + h * a.b_sh + (pos + s) * a.b_ss + d0;
  }
  uint4 xa = make_uint4(0, 0, 0, 0), xb = xa;
  if (src) {
    xa = ld_stream(src);
    xb = ld_stream(src + kHalfD);
  }
  if (is_v) {  // v rows: plain copy into the cache (no norm, no rotation)
    st_vec(dst, xa);
    st_vec(dst + kHalfD, xb);
  }
  float x[8], y[8];
  unpack8(xa, x);
  unpack8(xb, y);
  // per-head RMSNorm: all lanes of the group take part in the shuffles
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss += x[j] * x[j];
#pragma unroll
  for (int j = 0; j < 8; ++j) ss += y[j] * y[j];
#pragma unroll
  for (int o = TPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (!is_q && !is_k) return;
  const void* w = is_q ? a.qw : a.kw;
  if (w) {
    const float rstd = rsqrtf(ss / static_cast<float>(TPH * 16) + (is_q ? a.q_eps : a.k_eps));
    float wv[8];
    load_w8(w, a.w_dtype, d0, wv);
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = x[j] * rstd * wv[j];
    load_w8(w, a.w_dtype, d0 + kHalfD, wv);
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = y[j] * rstd * wv[j];
  }
  // rotate-half RoPE: out[d] = x[d] cos[d] - x[d + D/2] sin[d] for the first half,
  // out[d + D/2] = x[d + D/2] cos[d + D/2] + x[d] sin[d + D/2] for the second
  const int64_t crow = b * a.c_sb + s * a.c_ss + d0;
  float c[8], sn[8], o[8];
  load_table8<kCosFp32>(a.cos, crow, c);
  load_table8<kCosFp32>(a.sin, crow, sn);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = x[j] * c[j] - y[j] * sn[j];
  st_vec(dst, pack8(o));
  load_table8<kCosFp32>(a.cos, crow + kHalfD, c);
  load_table8<kCosFp32>(a.sin, crow + kHalfD, sn);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = y[j] * c[j] + x[j] * sn[j];
  st_vec(dst + kHalfD, pack8(o));
}

template <int TPH>
void launch_prep(const PrepArgs& a, int64_t seq, int64_t batch, int zblocks, bool cos32,
                 cudaStream_t st) {
  const dim3 grid(static_cast<unsigned>(seq), static_cast<unsigned>(batch),
                  static_cast<unsigned>(zblocks));
  if (cos32) {
    prefer_max_shared<qk_prep_kernel<TPH, true>>();
    launch_pdl(qk_prep_kernel<TPH, true>, grid, dim3(kPrepThreads), 0, st, a);
  } else {
    prefer_max_shared<qk_prep_kernel<TPH, false>>();
    launch_pdl(qk_prep_kernel<TPH, false>, grid, dim3(kPrepThreads), 0, st, a);
  }
}

}  // namespace
}  // namespace umic

using namespace umic;

extern "C" int umic_qk_norm_rope_kv(
    void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh, int32_t hq, void* k, int64_t k_sb,
    int64_t k_ss, int64_t k_sh, const void* v, int64_t v_sb, int64_t v_ss, int64_t v_sh,
    int32_t hk, const void* q_weight, const void* k_weight, int w_dtype, float q_eps,
    float k_eps, const void* cos, const void* sin, int64_t c_sb, int64_t c_ss, int cos_dtype,
    void* k_buf, void* v_buf, int64_t buf_sb, int64_t buf_sh, int64_t buf_ss, int64_t capacity,
    int64_t pos, const int64_t* dpos, int64_t batch, int64_t seq, int32_t head_dim,
    void* stream) {
  clear_error();
  if (hq <= 0 || hk <= 0 || batch < 0 || seq < 0)
    return fail(UMIC_ERR_INVALID_ARG, "umic_qk_norm_rope_kv: hq=%d hk=%d", hq, hk);
  if (batch == 0 || seq == 0) return UMIC_OK;
  if (!q || !k || !cos || !sin || (k_buf && (!v || !v_buf)))
    return fail(UMIC_ERR_INVALID_ARG, "umic_qk_norm_rope_kv: null pointer");
  if (head_dim != 64 && head_dim != 128 && head_dim != 256)
    return fail(UMIC_ERR_UNSUPPORTED, "umic_qk_norm_rope_kv: head_dim %d (64, 128 or 256)",
                head_dim);
  if (w_dtype != UMIC_DTYPE_BF16 && w_dtype != UMIC_DTYPE_FP32)
    return fail(UMIC_ERR_INVALID_ARG, "umic_qk_norm_rope_kv: bad w_dtype");
  if (cos_dtype != UMIC_DTYPE_BF16 && cos_dtype != UMIC_DTYPE_FP32)
    return fail(UMIC_ERR_INVALID_ARG, "umic_qk_norm_rope_kv: bad cos_dtype");
  const int64_t celem = cos_dtype == UMIC_DTYPE_FP32 ? 4 : 8;
  const bool aligned = aligned16(q) && aligned16(k) && aligned16(cos) && aligned16(sin) &&
                       (!v || aligned16(v)) && (!k_buf || (aligned16(k_buf) && aligned16(v_buf))) &&
                       q_sb % 8 == 0 && q_ss % 8 == 0 && q_sh % 8 == 0 && k_sb % 8 == 0 &&
                       k_ss % 8 == 0 && k_sh % 8 == 0 && v_sb % 8 == 0 && v_ss % 8 == 0 &&
                       v_sh % 8 == 0 && buf_sb % 8 == 0 && buf_sh % 8 == 0 &&
                       buf_ss % 8 == 0 && c_sb % celem == 0 && c_ss % celem == 0;
  if (!aligned)
    return fail(UMIC_ERR_ALIGNMENT, "umic_qk_norm_rope_kv: 16-byte alignment of bases/strides");
  const bool wq_al = !q_weight || (w_dtype == UMIC_DTYPE_FP32
                                       ? (reinterpret_cast<uintptr_t>(q_weight) & 31u) == 0
                                       : aligned16(q_weight));
  const bool wk_al = !k_weight || (w_dtype == UMIC_DTYPE_FP32
                                       ? (reinterpret_cast<uintptr_t>(k_weight) & 31u) == 0
                                       : aligned16(k_weight));
  if (!wq_al || !wk_al) return fail(UMIC_ERR_ALIGNMENT, "umic_qk_norm_rope_kv: norm weights");
  if (k_buf && !dpos && (pos < 0 || pos + seq > capacity))
    return fail(UMIC_ERR_OVERFLOW, "InplaceLayer overflow: pos %lld + new %lld > buffer %lld",
                (long long)pos, (long long)seq, (long long)capacity);
  if (batch > 65535 || seq > 0x7fffffffLL)
    return fail(UMIC_ERR_UNSUPPORTED, "umic_qk_norm_rope_kv: batch/seq too large");
  PrepArgs a{static_cast<__nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(k),
             static_cast<const __nv_bfloat16*>(v), q_weight, k_weight, cos, sin,
             static_cast<__nv_bfloat16*>(k_buf), static_cast<__nv_bfloat16*>(v_buf), dpos,
             device_error_word(), q_sb, q_ss, q_sh, k_sb, k_ss, k_sh, v_sb, v_ss, v_sh, c_sb,
             c_ss, buf_sb, buf_sh, buf_ss, capacity, pos, seq, hq, hk, w_dtype, q_eps,
             k_eps};
  const int tph = head_dim / 16;
  const int rows_per_block = kPrepThreads / tph;
  const int rows = hq + (k_buf ? 2 * hk : hk);
  const int zblocks = (rows + rows_per_block - 1) / rows_per_block;
  if (zblocks > 65535)
    return fail(UMIC_ERR_UNSUPPORTED, "umic_qk_norm_rope_kv: too many heads (%d + %d)", hq, hk);
  const bool cos32 = cos_dtype == UMIC_DTYPE_FP32;
  cudaStream_t st = as_stream(stream);
  if (tph == 4) launch_prep<4>(a, seq, batch, zblocks, cos32, st);
  else if (tph == 8) launch_prep<8>(a, seq, batch, zblocks, cos32, st);
  else launch_prep<16>(a, seq, batch, zblocks, cos32, st);
  return launch_status("umic_qk_norm_rope_kv");
}
